// allpairs.cu -- host scheduler of the all-pairs scoring call.
//
// Replaces the reference's per-pair loop (gafime/backends/native_cuda_backend.py:368-379:
// one launch + memset + D2H + sync per pair) and its Rust pair enumeration
// (src/cpu/gafime_cpu/src/batch_launcher.rs:216-247, smart_scheduler.rs:78-176) with:
//   1. fp64 column statistics (bucket.cu), once per call;
//   2. upper-triangle 64 x 64 pair tiles, assigned to shards by tile work and column reads;
//   3. split-K over rows so every SM has work, fp64 partials per (tile, split);
//   4. the scoring epilogue with a per-tile bitonic top-k, one launch per operator;
//   5. a device merge of the per-tile lists and one small D2H per operator.
// Everything is queued on the bucket's stream; the only host sync is the final copy.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "engine.h"

namespace gafime {

namespace {

int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

int64_t tile_pairs(int bi, int bj, int64_t f) {
    int64_t i0 = (int64_t)bi * kTile, j0 = (int64_t)bj * kTile;
    int64_t ni = std::min<int64_t>(kTile, f - i0), nj = std::min<int64_t>(kTile, f - j0);
    if (ni <= 0 || nj <= 0) return 0;
    if (bi != bj) return ni * nj;
    return ni * (ni - 1) / 2;
}

}  // namespace

// Upper-triangle 64 x 64 tiles of this shard.  The pair space is dealt out in
// 128 x 128 blocks (the tensor-core Gram tile): blocks in decreasing work (ties in
// row-major order), each to the shard with the least work so far (ties: lowest shard id);
// a shard scores the 64-tiles inside its blocks.  A block's work is the number of 64-tiles
// it holds (4 off the diagonal, 3 on it), not its pair count: a tile costs the same
// whether its pairs are distinct or mirrored, and a diagonal 128-tile on the Gram path
// measured ~0.8 of an off-diagonal one (0.5 by pair count, which left the shards that
// held the diagonal 5-9 % slower).  Every process derives the same split without
// communication.
static std::vector<TileCoord> compute_shard_tiles(int64_t f, int shard_id, int n_shards) {
    int nb = (int)((f + kTile - 1) / kTile);
    int nb2 = (nb + 1) / 2;
    struct Block {
        int64_t w;
        int order, ns;
        TileCoord sub[4];
        int BI, BJ;   // its two 128-column blocks
    };
    std::vector<Block> blocks;
    for (int BI = 0; BI < nb2; ++BI)
        for (int BJ = BI; BJ < nb2; ++BJ) {
            Block blk{0, (int)blocks.size(), 0, {}, BI, BJ};
            for (int da = 0; da < 2; ++da)
                for (int db = 0; db < 2; ++db) {
                    int bi = 2 * BI + da, bj = 2 * BJ + db;
                    if (bi > bj || bi >= nb || bj >= nb) continue;
                    if (tile_pairs(bi, bj, f) == 0) continue;
                    blk.sub[blk.ns++] = {bi, bj};
                    blk.w += 1;   // work: one 64-tile
                }
            if (blk.w > 0) blocks.push_back(blk);
        }
    std::stable_sort(blocks.begin(), blocks.end(),
                     [](const Block& x, const Block& y) { return x.w > y.w; });
    std::vector<int64_t> load((size_t)n_shards, 0);
    std::vector<int> owner(blocks.size());
    for (size_t x = 0; x < blocks.size(); ++x) {
        int best = 0;
        for (int s = 1; s < n_shards; ++s)
            if (load[(size_t)s] < load[(size_t)best]) best = s;
        load[(size_t)best] += blocks[x].w;
        owner[x] = best;
    }
    // Locality: a shard prepares the 128-column blocks its tiles read, so swap blocks of equal
    // work between two shards while that lowers the larger, then the summed, number of
    // column blocks the two read (the loads do not change).  Fixed scan order: every process
    // arrives at the same assignment.  Per-shard counts of the owned blocks touching each
    // column block make a trial swap O(1); skipped for very wide matrices.
    if (n_shards > 1 && blocks.size() <= 2048) {
        std::vector<int> cnt((size_t)n_shards * nb2, 0), reads((size_t)n_shards, 0);
        // multiplicities: a diagonal block counts its column block twice, consistently
        auto add = [&](int s, int x, int d) {
            for (int B : {blocks[(size_t)x].BI, blocks[(size_t)x].BJ}) {
                int& c = cnt[(size_t)s * nb2 + B];
                if (d > 0 && c++ == 0) ++reads[(size_t)s];
                if (d < 0 && --c == 0) --reads[(size_t)s];
            }
        };
        for (size_t x = 0; x < blocks.size(); ++x) add(owner[x], (int)x, +1);
        for (int pass = 0; pass < 64; ++pass) {
            bool swapped = false;
            for (int a = 0; a < n_shards && !swapped; ++a)
                for (int b = a + 1; b < n_shards && !swapped; ++b) {
                    const int ra = reads[(size_t)a], rb = reads[(size_t)b];
                    for (size_t x = 0; x < blocks.size() && !swapped; ++x) {
                        if (owner[x] != a) continue;
                        for (size_t y = 0; y < blocks.size() && !swapped; ++y) {
                            if (owner[y] != b || blocks[y].w != blocks[x].w) continue;
                            // trial swap
                            add(a, (int)x, -1);
                            add(b, (int)y, -1);
                            add(a, (int)y, +1);
                            add(b, (int)x, +1);
                            const int na = reads[(size_t)a], nbr = reads[(size_t)b];
                            if (std::max(na, nbr) < std::max(ra, rb) ||
                                (std::max(na, nbr) == std::max(ra, rb) && na + nbr < ra + rb)) {
                                owner[x] = b;
                                owner[y] = a;
                                swapped = true;
                            } else {
                                add(a, (int)y, -1);
                                add(b, (int)x, -1);
                                add(a, (int)x, +1);
                                add(b, (int)y, +1);
                            }
                        }
                    }
                }
            if (!swapped) break;
        }
    }
    // A shard's time is its tile work plus the preparation of every 128-column block its
    // tiles read (statistics and operand scales over all rows of the block): per 64-tile
    // ~0.2 ms and per block ~0.15 ms at 2e6 rows on the Gram path, both proportional to the
    // rows.  cost = 4 work + 3 reads; a plan costs its busiest shard's cost.
    if (n_shards > 1) {
        auto plan_cost = [&](const std::vector<int>& own, int64_t* max_cost, int* max_reads) {
            std::vector<int64_t> ld((size_t)n_shards, 0);
            std::vector<std::vector<char>> rd((size_t)n_shards, std::vector<char>((size_t)nb2, 0));
            for (size_t x = 0; x < blocks.size(); ++x) {
                ld[(size_t)own[x]] += blocks[x].w;
                rd[(size_t)own[x]][(size_t)blocks[x].BI] = rd[(size_t)own[x]][(size_t)blocks[x].BJ] = 1;
            }
            *max_cost = 0;
            *max_reads = 0;
            for (int sh = 0; sh < n_shards; ++sh) {
                int r = 0;
                for (char c : rd[(size_t)sh]) r += c;
                *max_cost = std::max(*max_cost, 4 * ld[(size_t)sh] + 3 * (int64_t)r);
                *max_reads = std::max(*max_reads, r);
            }
        };
        // Grouped alternatives: split the 128-column blocks into g contiguous groups; a unit is
        // every block of one group pair (Ga, Gb), a <= b, so a shard owning units of few
        // groups reads few column blocks.  Units in decreasing work go to the least-loaded
        // shard (ties: lowest id).  The cheapest plan is kept (ties: the earlier one).
        const std::vector<int> greedy = owner;
        std::vector<int> grouped;
        std::vector<std::vector<int>> starts;   // every grouped plan, searched when few blocks
        const bool search_all = blocks.size() <= 512;
        int64_t best_cost = INT64_MAX;
        int best_reads = 0;
        for (int g = 2; g <= nb2; ++g) {
            if ((int64_t)g * (g + 1) / 2 < n_shards) continue;
            std::vector<int> grp((size_t)nb2);
            for (int B = 0; B < nb2; ++B) grp[(size_t)B] = (int)((int64_t)B * g / nb2);
            const int units = g * (g + 1) / 2;
            std::vector<int64_t> uw((size_t)units, 0);
            auto uid = [&](int ga, int gb) { return ga * g - ga * (ga - 1) / 2 + (gb - ga); };
            for (const Block& blk : blocks) uw[(size_t)uid(grp[(size_t)blk.BI], grp[(size_t)blk.BJ])] += blk.w;
            std::vector<int> order((size_t)units);
            for (int u = 0; u < units; ++u) order[(size_t)u] = u;
            std::stable_sort(order.begin(), order.end(),
                             [&](int x, int y) { return uw[(size_t)x] > uw[(size_t)y]; });
            std::vector<int64_t> sl((size_t)n_shards, 0);
            std::vector<int> uown((size_t)units, 0);
            for (int u : order) {
                int bs = 0;
                for (int sh = 1; sh < n_shards; ++sh)
                    if (sl[(size_t)sh] < sl[(size_t)bs]) bs = sh;
                sl[(size_t)bs] += uw[(size_t)u];
                uown[(size_t)u] = bs;
            }
            std::vector<int> own(blocks.size());
            for (size_t x = 0; x < blocks.size(); ++x)
                own[x] = uown[(size_t)uid(grp[(size_t)blocks[x].BI], grp[(size_t)blocks[x].BJ])];
            int64_t mc = 0;
            int mr = 0;
            plan_cost(own, &mc, &mr);
            if (search_all) starts.push_back(own);
            if (mc < best_cost || (mc == best_cost && mr < best_reads)) {
                grouped = own;
                best_cost = mc;
                best_reads = mr;
            }
        }
        // Local search: move a block off the costliest shard (lowest id on ties) to the shard
        // where the larger of the two new costs is smallest, or swap two blocks, while that
        // lowers the costliest shard's cost.  Run from the greedy plan and from every grouped
        // plan (only the cheapest grouped one above 512 blocks); the cheapest result is kept
        // (ties: fewer column blocks, then the earlier start).  Fixed scan order: every process
        // arrives at the same plan.
        auto improve = [&](std::vector<int>& own) {
            if (blocks.size() > 4096) return;
            std::vector<int> cnt((size_t)n_shards * nb2, 0), reads((size_t)n_shards, 0);
            std::vector<int64_t> work((size_t)n_shards, 0);
            auto add = [&](int sh, int x, int d) {
                work[(size_t)sh] += d * blocks[(size_t)x].w;
                for (int B : {blocks[(size_t)x].BI, blocks[(size_t)x].BJ}) {
                    int& c = cnt[(size_t)sh * nb2 + B];
                    if (d > 0 && c++ == 0) ++reads[(size_t)sh];
                    if (d < 0 && --c == 0) --reads[(size_t)sh];
                }
            };
            auto cost = [&](int sh) { return 4 * work[(size_t)sh] + 3 * (int64_t)reads[(size_t)sh]; };
            for (size_t x = 0; x < blocks.size(); ++x) add(own[x], (int)x, +1);
            for (size_t it = 0; it < 4 * blocks.size(); ++it) {
                int m = 0;
                for (int sh = 1; sh < n_shards; ++sh)
                    if (cost(sh) > cost(m)) m = sh;
                const int64_t cm = cost(m);
                int64_t best = cm;
                int bx = -1, by = -1, bt = -1;
                for (size_t x = 0; x < blocks.size(); ++x) {
                    if (own[x] != m) continue;
                    for (int t = 0; t < n_shards; ++t) {
                        if (t == m) continue;
                        add(m, (int)x, -1);
                        add(t, (int)x, +1);
                        const int64_t c = std::max(cost(m), cost(t));
                        if (c < best) { best = c; bx = (int)x; by = -1; bt = t; }
                        add(t, (int)x, -1);
                        add(m, (int)x, +1);
                    }
                }
                if (bx < 0) {   // swaps, only when no single move helps
                    for (size_t x = 0; x < blocks.size() && bx < 0; ++x) {
                        if (own[x] != m) continue;
                        for (size_t y = 0; y < blocks.size(); ++y) {
                            const int t = own[y];
                            if (t == m || blocks[y].w >= blocks[x].w) continue;
                            add(m, (int)x, -1);
                            add(t, (int)y, -1);
                            add(m, (int)y, +1);
                            add(t, (int)x, +1);
                            const int64_t c = std::max(cost(m), cost(t));
                            add(t, (int)x, -1);
                            add(m, (int)y, -1);
                            add(t, (int)y, +1);
                            add(m, (int)x, +1);
                            if (c < best) { best = c; bx = (int)x; by = (int)y; bt = t; }
                        }
                    }
                }
                if (bx < 0) break;
                add(m, bx, -1);
                add(bt, bx, +1);
                own[(size_t)bx] = bt;
                if (by >= 0) {
                    add(bt, by, -1);
                    add(m, by, +1);
                    own[(size_t)by] = m;
                }
            }
        };
        if (!search_all && !grouped.empty()) starts.push_back(grouped);
        owner = greedy;
        improve(owner);
        int64_t cbest = 0;
        int rbest = 0;
        plan_cost(owner, &cbest, &rbest);
        for (std::vector<int>& st : starts) {
            improve(st);
            int64_t c = 0;
            int r = 0;
            plan_cost(st, &c, &r);
            if (c < cbest || (c == cbest && r < rbest)) {
                owner = st;
                cbest = c;
                rbest = r;
            }
        }
    }
    std::vector<TileCoord> mine;
    for (size_t x = 0; x < blocks.size(); ++x)
        if (owner[x] == shard_id)
            for (int q = 0; q < blocks[x].ns; ++q) mine.push_back(blocks[x].sub[q]);
    return mine;
}

// The assignment depends on (f, shard_id, n_shards) only: computed once per process and kept.
std::vector<TileCoord> shard_tiles(int64_t f, int shard_id, int n_shards) {
    static std::mutex mu;
    static std::map<std::tuple<int64_t, int, int>, std::vector<TileCoord>> memo;
    const auto key = std::make_tuple(f, shard_id, n_shards);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = memo.find(key);
        if (it != memo.end()) return it->second;
    }
    std::vector<TileCoord> t = compute_shard_tiles(f, shard_id, n_shards);
    std::lock_guard<std::mutex> lock(mu);
    if (memo.size() > 256) memo.clear();
    memo[key] = t;
    return t;
}

namespace {

struct Plan {
    std::vector<TileCoord> tiles;
    int splits = 1;
    int64_t rows_per_split = 0;
};

Plan make_plan(const Bucket& b, int shard_id, int n_shards) {
    Plan p;
    p.tiles = shard_tiles(b.f, shard_id, n_shards);
    // row splits from the whole matrix's tile count (not this shard's), so a pair's partial
    // sums cover the same rows on every shard count
    const int64_t nb = (b.f + kTile - 1) / kTile;
    const int64_t all_tiles = std::max<int64_t>(1, nb * (nb + 1) / 2);
    int splits = (int)std::max<int64_t>(1, b.sm_count / all_tiles);
    // at least 1024 rows per split
    int64_t max_splits = std::max<int64_t>(1, b.ld / 1024);
    if (splits > max_splits) splits = (int)max_splits;
    int64_t rps = (b.ld + splits - 1) / splits;
    rps = (rps + kRowPad - 1) / kRowPad * kRowPad;
    p.splits = (int)((b.ld + rps - 1) / rps);
    p.rows_per_split = rps;
    return p;
}

bool valid_op(int op) { return op >= GAFIME_INTERACT_MULT && op <= GAFIME_INTERACT_DIV; }
bool valid_metric(int m) {
    return m == GAFIME_METRIC_PEARSON || m == GAFIME_METRIC_MUTUAL_INFO || m == GAFIME_METRIC_MUTUAL_INFO_QUANTILE;
}

// Column statistics for one call.  Mutual information centres on the fly from the
// raw-column means, so it always asks for uncentred statistics.
// pair_scoring: the caller scores pairs next, so on the tensor-core path (raw Pearson) the
// column sums come from the Gram statistics pass instead of a pass of their own.
int prepare(Bucket& b, int center, int metric, ColumnStats& cs, bool pair_scoring) {
    bool finite = true;
    int st = check_finite(b, &finite);  // computed at upload; a cached flag here
    if (st != GAFIME_SUCCESS) return st;
    if (!finite) return GAFIME_ERROR_INVALID_ARGS;
    const bool centred = center != 0 && metric == GAFIME_METRIC_PEARSON;
    const bool gram_sums = pair_scoring && metric == GAFIME_METRIC_PEARSON && !centred && gram_path_enabled(b);
    KernelTimer timer(b.stream, GAFIME_KERNEL_COLUMN_STATS);
    return compute_column_stats(b, centred, cs, !gram_sums);
}

// Pearson per pair of every operator from the moments of its group (0: multiply / add /
// subtract, 1: divide) and the per-list top-k (or every score into all_scores).
// Before it, the accuracy guard flags the pairs whose moments may have lost the 1e-4
// bound and re-scores them exactly (guard.cu); gram: the moments come from the tensor-core
// Gram path.
int queue_epilogue(Bucket& b, const ColumnStats& cs, const TileCoord* d_tiles, int nt, const int* ops, int n_ops,
                   const double* mom_mul, int splits_mul, const double* mom_div, int splits_div, int k_pad,
                   int sub_lists, Cand* const* cands, double* all_scores, float div_eps, bool gram) {
    EpilogueArgs a;
    memset(&a, 0, sizeof(a));
    for (int o = 0; o < n_ops; ++o) {
        const bool div = ops[o] == GAFIME_INTERACT_DIV;
        a.moments[o] = div ? mom_div : mom_mul;
        a.splits[o] = div ? splits_div : splits_mul;
        a.op[o] = ops[o];
        a.cands[o] = cands[o];
    }
    a.n_ops = n_ops;
    a.tiles = d_tiles;
    a.n_tiles = nt;
    a.f = b.f;
    a.colstats = cs.d_col;
    a.ystats = cs.d_y;
    a.k_pad = k_pad;
    a.sub_lists = sub_lists;
    a.all_scores = all_scores;
    cudaError_t e;
    {
        // guard scratch: the re-score counter (first, where queue_rescored_read finds it),
        // flags (bytes), exact scores and the re-score list
        const size_t pairs = (size_t)n_ops * nt * kTilePairs;
        const size_t off_count = 0, off_flags = 256;
        const size_t off_exact = (off_flags + pairs + 255) / 256 * 256;
        const size_t off_list = off_exact + pairs * sizeof(double);
        e = ensure(b.guard, off_list + pairs * sizeof(uint2));
        if (e != cudaSuccess) return status_from(e);
        char* base = (char*)b.guard.ptr;
        GuardArgs g;
        memset(&g, 0, sizeof(g));
        RescoreArgs r;
        memset(&r, 0, sizeof(r));
        for (int o = 0; o < n_ops; ++o) {
            g.moments[o] = a.moments[o];
            g.splits[o] = a.splits[o];
            g.op[o] = r.op[o] = ops[o];
        }
        g.n_ops = n_ops;
        g.tiles = r.tiles = d_tiles;
        g.n_tiles = r.n_tiles = nt;
        g.f = b.f;
        g.colstats = cs.d_col;
        g.ystats = r.ystats = cs.d_y;
        g.gram = gram ? 1 : 0;
        g.gstats = gram ? gram_col_state(b) : nullptr;
        g.flags = (uint8_t*)(base + off_flags);
        g.count = (unsigned long long*)(base + off_count);
        g.list = (uint2*)(base + off_list);
        r.x = cs.d_x;
        r.y = b.d_data + b.f * b.ld;
        r.ld = b.ld;
        r.n = b.n;
        r.eps = div_eps;
        r.count = g.count;
        r.list = g.list;
        r.exact = (double*)(base + off_exact);
        a.guard_flags = g.flags;
        a.exact = r.exact;
        KernelTimer timer(b.stream, GAFIME_KERNEL_GUARD);
        e = launch_guard(g, r, b.sm_count, b.stream);
        if (e != cudaSuccess) return status_from(e);
        b.guard_ran = true;
    }
    {
        KernelTimer timer(b.stream, GAFIME_KERNEL_EPILOGUE_TOPK);
        e = launch_epilogue_topk(a, b.stream);
    }
    return status_from(e);
}

// Queue moments + epilogue for the requested operators.  cands[o] receives n_tiles *
// sub_lists lists of k_pad entries for operator o (nullptr: no selection); mutual
// information writes n_tiles lists.
int score_ops(Bucket& b, const ColumnStats& cs, const Plan& plan, const TileCoord* d_tiles,
              const int* ops, int n_ops, int metric, int center, float div_eps, int mi_bins,
              int k_pad, int sub_lists, Cand* const* cands, double* all_scores, int* gram_used) {
    *gram_used = 0;
    const int nt = (int)plan.tiles.size();
    if (nt == 0) return GAFIME_SUCCESS;
    cudaError_t e;
    if (metric == GAFIME_METRIC_MUTUAL_INFO_QUANTILE) {
        for (int o = 0; o < n_ops; ++o) {
            e = launch_mi_quantile(b, cs, center != 0, ops[o], div_eps, mi_bins, plan.tiles, d_tiles, k_pad,
                                   cands[o], all_scores, b.stream);
            if (e != cudaSuccess) return status_from(e);
        }
        return GAFIME_SUCCESS;
    }
    if (metric == GAFIME_METRIC_MUTUAL_INFO) {
        for (int o = 0; o < n_ops; ++o) {
            e = launch_mi_scores(b, cs, center != 0, ops[o], div_eps, mi_bins, d_tiles, nt, k_pad,
                                 cands[o], all_scores, b.stream);
            if (e != cudaSuccess) return status_from(e);
        }
        return GAFIME_SUCCESS;
    }
    size_t group_bytes = (size_t)plan.splits * nt * 3 * kTilePairs * sizeof(double);
    e = ensure(b.moments, 2 * group_bytes);
    if (e != cudaSuccess) return status_from(e);
    double* mom[2] = {(double*)b.moments.ptr, (double*)((char*)b.moments.ptr + group_bytes)};
    bool need[2] = {false, false};
    int group_splits[2] = {plan.splits, plan.splits};
    for (int o = 0; o < n_ops; ++o) need[ops[o] == GAFIME_INTERACT_DIV ? 1 : 0] = true;
    const bool tensor = gram_path_enabled(b);
    if (tensor) {
        // the Gram kernels' error flag is read once by the caller after its final copy
        e = gram_error_reset(b, b.stream);
        if (e != cudaSuccess) return status_from(e);
        *gram_used = 1;
    }
    for (int g = 0; g < 2; ++g) {
        if (!need[g]) continue;
        if (tensor) {
            // one operand preparation serves both groups when both are scored
            const int prep = (g == 0 && need[1]) ? GRAM_PREP_BOTH : (g == 1 && need[0]) ? GRAM_PREP_DONE
                                                                                      : GRAM_PREP_OWN;
            e = launch_gram_moments(b, cs, d_tiles, plan.tiles, g == 1, div_eps, mom[g], b.stream, nullptr,
                                    prep);
            if (e != cudaSuccess) return status_from(e);
            group_splits[g] = 1;
        } else {
            KernelTimer timer(b.stream, GAFIME_KERNEL_PAIR_MOMENTS);
            e = launch_pair_moments(cs.d_x, b.ld, cs.d_ycen, b.f, d_tiles, nt, plan.splits,
                                    plan.rows_per_split, g == 1, div_eps, mom[g], b.stream);
            if (e != cudaSuccess) return status_from(e);
        }
    }
    return queue_epilogue(b, cs, d_tiles, nt, ops, n_ops, mom[0], group_splits[0], mom[1], group_splits[1], k_pad,
                          sub_lists, cands, all_scores, div_eps, tensor);
}

int merge_and_copy(Bucket& b, Cand* const* cands, Cand* const* tmp, int n_lists, int k, int k_pad, int n_ops,
                   size_t per_op, int32_t* out_i, int32_t* out_j, double* out_score, int* out_count);

// The guard's re-score count of this call: copied into the bucket's pinned staging on its
// stream (queue), read after the caller's synchronize (finish).  MI calls run no guard and
// leave the counter untouched, so they report 0.
cudaError_t queue_rescored_read(Bucket& b) {
    unsigned long long* h = reinterpret_cast<unsigned long long*>(b.h_pinned + 63);
    *h = 0;
    if (!b.guard_ran) return cudaSuccess;
    return cudaMemcpyAsync(h, b.guard.ptr, sizeof(unsigned long long), cudaMemcpyDeviceToHost, b.stream);
}

void finish_rescored_read(Bucket& b) {
    b.last_rescored += (int64_t)*reinterpret_cast<unsigned long long*>(b.h_pinned + 63);
}

// GAFIME_ERROR_KERNEL_FAILED when a Gram kernel of this call recorded a wait timeout
int gram_status(Bucket& b, int gram_used) {
    if (!gram_used) return GAFIME_SUCCESS;
    int err = 0;
    cudaError_t e = gram_error_read(b, b.stream, &err);
    if (e != cudaSuccess) return status_from(e);
    return err ? GAFIME_ERROR_KERNEL_FAILED : GAFIME_SUCCESS;
}

int upload_tiles(Bucket& b, const Plan& plan, TileCoord** d_tiles) {
    size_t bytes = std::max<size_t>(1, plan.tiles.size()) * sizeof(TileCoord);
    cudaError_t e = ensure(b.tiles, bytes);
    if (e != cudaSuccess) return status_from(e);
    if (!plan.tiles.empty()) {
        e = cudaMemcpyAsync(b.tiles.ptr, plan.tiles.data(), plan.tiles.size() * sizeof(TileCoord),
                            cudaMemcpyHostToDevice, b.stream);
        if (e != cudaSuccess) return status_from(e);
    }
    *d_tiles = (TileCoord*)b.tiles.ptr;
    return GAFIME_SUCCESS;
}

}  // namespace

}  // namespace gafime

using namespace gafime;

namespace gafime {
namespace {

int check_topk_args(ContiguousBucket bucket, const int* interact_types, int n_ops, int metric, float div_eps,
                    int mi_bins, int k, int shard_id, int n_shards) {
    if (!bucket || !interact_types || n_ops < 1 || n_ops > 4 || k < 1 || k > GAFIME_ALLPAIRS_MAX_K ||
        n_shards < 1 || shard_id < 0 || shard_id >= n_shards)
        return GAFIME_ERROR_INVALID_ARGS;
    if (!valid_metric(metric)) return GAFIME_ERROR_INVALID_ARGS;
    if (metric != GAFIME_METRIC_PEARSON && (mi_bins < 2 || mi_bins > 255)) return GAFIME_ERROR_INVALID_ARGS;
    if (!(div_eps > 0.0f)) return GAFIME_ERROR_INVALID_ARGS;
    for (int o = 0; o < n_ops; ++o)
        if (!valid_op(interact_types[o])) return GAFIME_ERROR_INVALID_ARGS;
    if (((Bucket*)bucket)->f >= 65536) return GAFIME_ERROR_INVALID_ARGS;  // pair id i*F + j must fit 32 bits
    return GAFIME_SUCCESS;
}

// The scoring of one top-k call, queued on the bucket's stream without a host sync: the
// per-list candidates of every operator land in cands[o] (n_lists lists of k_pad entries;
// tmp[o] is the merge's second buffer).  nt == 0 (no tile in this shard) queues nothing.
struct TopkQueued {
    Cand* cands[4];
    Cand* tmp[4];
    int n_lists = 0, k_pad = 1, nt = 0, gram_used = 0;
    size_t per_op = 0;
};

int queue_topk(Bucket& b, const int* ops, int n_ops, int metric, int center, float div_eps, int mi_bins, int k,
               int shard_id, int n_shards, TopkQueued& q) {
    b.last_rescored = 0;
    b.guard_ran = false;
    Plan plan = make_plan(b, shard_id, n_shards);
    q.nt = (int)plan.tiles.size();
    q.k_pad = next_pow2(k);
    if (q.nt == 0) return GAFIME_SUCCESS;
    ColumnStats cs;
    int st = prepare(b, center, metric, cs, true);
    if (st != GAFIME_SUCCESS) return st;
    TileCoord* d_tiles = nullptr;
    st = upload_tiles(b, plan, &d_tiles);
    if (st != GAFIME_SUCCESS) return st;
    const int sub_lists = metric == GAFIME_METRIC_PEARSON ? epilogue_sub_lists(q.nt, q.k_pad, b.sm_count) : 1;
    q.n_lists = q.nt * sub_lists;
    q.per_op = (size_t)q.n_lists * q.k_pad;
    cudaError_t e = ensure(b.cands, q.per_op * n_ops * sizeof(Cand));
    if (e == cudaSuccess) e = ensure(b.cands2, q.per_op * n_ops * sizeof(Cand));
    if (e != cudaSuccess) return status_from(e);
    for (int o = 0; o < n_ops; ++o) {
        q.cands[o] = (Cand*)b.cands.ptr + q.per_op * o;
        q.tmp[o] = (Cand*)b.cands2.ptr + q.per_op * o;
    }
    return score_ops(b, cs, plan, d_tiles, ops, n_ops, metric, center, div_eps, mi_bins, q.k_pad, sub_lists,
                     q.cands, nullptr, &q.gram_used);
}

}  // namespace
}  // namespace gafime

extern "C" int gafime_allpairs_topk(ContiguousBucket bucket, const int* interact_types, int n_ops,
                                    int metric, int center, float div_eps, int mi_bins, int k,
                                    int shard_id, int n_shards, int32_t* out_i, int32_t* out_j,
                                    double* out_score, int* out_count) {
    int st = check_topk_args(bucket, interact_types, n_ops, metric, div_eps, mi_bins, k, shard_id, n_shards);
    if (st != GAFIME_SUCCESS) return st;
    if (!out_i || !out_j || !out_score || !out_count) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    cudaSetDevice(b.device);
    for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
    TopkQueued q;
    st = queue_topk(b, interact_types, n_ops, metric, center, div_eps, mi_bins, k, shard_id, n_shards, q);
    if (st != GAFIME_SUCCESS || q.nt == 0) return st;
    st = merge_and_copy(b, q.cands, q.tmp, q.n_lists, k, q.k_pad, n_ops, q.per_op, out_i, out_j, out_score,
                        out_count);
    if (st == GAFIME_SUCCESS) st = gram_status(b, q.gram_used);
    if (st != GAFIME_SUCCESS)
        for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
    return st;
}

extern "C" int gafime_allpairs_topk_device(ContiguousBucket bucket, const int* interact_types, int n_ops,
                                           int metric, int center, float div_eps, int mi_bins, int k,
                                           int shard_id, int n_shards, void* d_cands) {
    int st = check_topk_args(bucket, interact_types, n_ops, metric, div_eps, mi_bins, k, shard_id, n_shards);
    if (st != GAFIME_SUCCESS) return st;
    if (!d_cands || ((uintptr_t)d_cands & 15) != 0) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    cudaSetDevice(b.device);
    TopkQueued q;
    st = queue_topk(b, interact_types, n_ops, metric, center, div_eps, mi_bins, k, shard_id, n_shards, q);
    if (st != GAFIME_SUCCESS) return st;
    b.pending_gram = q.gram_used;
    Cand* out = static_cast<Cand*>(d_cands);
    cudaError_t e;
    if (q.nt == 0) {
        // no tile on this shard: empty lists (score 0, no pair) for the exchange
        e = fill_empty_lists(out, (size_t)n_ops * q.k_pad, b.stream);
    } else {
        Cand* fin = nullptr;
        {
            KernelTimer timer(b.stream, GAFIME_KERNEL_MERGE);
            e = merge_candidates(q.cands[0], q.tmp[0], q.n_lists, q.k_pad, n_ops, q.per_op, &fin, b.stream);
        }
        for (int o = 0; o < n_ops && e == cudaSuccess; ++o)
            e = cudaMemcpyAsync(out + (size_t)o * q.k_pad, fin + q.per_op * o, sizeof(Cand) * q.k_pad,
                                cudaMemcpyDeviceToDevice, b.stream);
    }
    return status_from(e);
}

extern "C" int gafime_topk_merge_device(ContiguousBucket bucket, const void* d_gathered, int n_shards, int n_ops,
                                        int k, int32_t* out_i, int32_t* out_j, double* out_score,
                                        int* out_count) {
    if (!bucket || !d_gathered || ((uintptr_t)d_gathered & 15) != 0 || n_shards < 1 || n_ops < 1 || n_ops > 4 ||
        k < 1 || k > GAFIME_ALLPAIRS_MAX_K || !out_i || !out_j || !out_score || !out_count)
        return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    cudaSetDevice(b.device);
    for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
    const int k_pad = next_pow2(k);
    const size_t per_op = (size_t)n_shards * k_pad;
    cudaError_t e = ensure(b.cands, per_op * n_ops * sizeof(Cand));
    if (e == cudaSuccess) e = ensure(b.cands2, per_op * n_ops * sizeof(Cand));
    if (e != cudaSuccess) return status_from(e);
    Cand* cands[4];
    Cand* tmp[4];
    for (int o = 0; o < n_ops; ++o) {
        cands[o] = (Cand*)b.cands.ptr + per_op * o;
        tmp[o] = (Cand*)b.cands2.ptr + per_op * o;
    }
    // [shard][op][k_pad] (the all-gather's order) -> [op][shard][k_pad] (the merge's)
    e = reorder_shard_lists(static_cast<const Cand*>(d_gathered), cands[0], n_shards, n_ops, k_pad, b.stream);
    if (e != cudaSuccess) return status_from(e);
    int st = merge_and_copy(b, cands, tmp, n_shards, k, k_pad, n_ops, per_op, out_i, out_j, out_score, out_count);
    if (st == GAFIME_SUCCESS) st = gram_status(b, b.pending_gram);
    b.pending_gram = 0;
    if (st != GAFIME_SUCCESS)
        for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
    return st;
}

namespace gafime {
namespace {

// Merge the per-list candidates of every operator, copy the k best to the host and write
// them in the output layout of gafime_allpairs_topk.
int merge_and_copy(Bucket& b, Cand* const* cands, Cand* const* tmp, int n_lists, int k, int k_pad, int n_ops,
                   size_t per_op, int32_t* out_i, int32_t* out_j, double* out_score, int* out_count) {
    std::vector<Cand> host((size_t)k_pad * n_ops);
    Cand* fin = nullptr;
    cudaError_t e;
    {
        KernelTimer timer(b.stream, GAFIME_KERNEL_MERGE);
        e = merge_candidates(cands[0], tmp[0], n_lists, k_pad, n_ops, per_op, &fin, b.stream);
    }
    if (e != cudaSuccess) return status_from(e);
    for (int o = 0; o < n_ops; ++o) {
        e = cudaMemcpyAsync(host.data() + (size_t)k_pad * o, fin + per_op * o, sizeof(Cand) * k_pad,
                            cudaMemcpyDeviceToHost, b.stream);
        if (e != cudaSuccess) return status_from(e);
    }
    e = queue_rescored_read(b);
    if (e != cudaSuccess) return status_from(e);
    e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return status_from(e);
    finish_rescored_read(b);
    for (int o = 0; o < n_ops; ++o) {
        int cnt = 0;
        for (int c = 0; c < k; ++c) {
            const Cand& cd = host[(size_t)k_pad * o + c];
            if (cd.pid == kNoPair) break;
            out_i[(size_t)o * k + c] = (int32_t)(cd.pid / (uint32_t)b.f);
            out_j[(size_t)o * k + c] = (int32_t)(cd.pid % (uint32_t)b.f);
            out_score[(size_t)o * k + c] = cd.score;
            ++cnt;
        }
        for (int c = cnt; c < k; ++c) {
            out_i[(size_t)o * k + c] = -1;
            out_j[(size_t)o * k + c] = -1;
            out_score[(size_t)o * k + c] = 0.0;
        }
        out_count[o] = cnt;
    }
    return GAFIME_SUCCESS;
}

}  // namespace
}  // namespace gafime

extern "C" int gafime_allpairs_scores(ContiguousBucket bucket, int interact_type, int metric,
                                      int center, float div_eps, int mi_bins, double* out_scores) {
    if (!bucket || !out_scores || !valid_op(interact_type)) return GAFIME_ERROR_INVALID_ARGS;
    if (!valid_metric(metric)) return GAFIME_ERROR_INVALID_ARGS;
    if (metric != GAFIME_METRIC_PEARSON && (mi_bins < 2 || mi_bins > 255)) return GAFIME_ERROR_INVALID_ARGS;
    if (!(div_eps > 0.0f)) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    if (b.f >= 65536) return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(b.device);
    b.last_rescored = 0;
    b.guard_ran = false;
    int64_t P = b.f * (b.f - 1) / 2;
    if (P == 0) return GAFIME_SUCCESS;
    Plan plan = make_plan(b, 0, 1);
    ColumnStats cs;
    int st = prepare(b, center, metric, cs, true);
    if (st != GAFIME_SUCCESS) return st;
    TileCoord* d_tiles = nullptr;
    st = upload_tiles(b, plan, &d_tiles);
    if (st != GAFIME_SUCCESS) return st;
    cudaError_t e = ensure(b.scores, (size_t)P * sizeof(double));
    if (e != cudaSuccess) return status_from(e);
    Cand* none[1] = {nullptr};
    int gram_used = 0;
    st = score_ops(b, cs, plan, d_tiles, &interact_type, 1, metric, center, div_eps, mi_bins, 1, 1,
                   none, (double*)b.scores.ptr, &gram_used);
    if (st != GAFIME_SUCCESS) return st;
    e = cudaMemcpyAsync(out_scores, b.scores.ptr, (size_t)P * sizeof(double), cudaMemcpyDeviceToHost,
                        b.stream);
    if (e == cudaSuccess && metric == GAFIME_METRIC_PEARSON) e = queue_rescored_read(b);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return status_from(e);
    if (metric == GAFIME_METRIC_PEARSON) finish_rescored_read(b);
    return gram_status(b, gram_used);
}

namespace gafime {
namespace {

// gafime_core pearson_from_sums (gafime_core.cpp:179-198) on raw-column sums:
// r = sum x*ycen / sqrt(var_x * var_y), var_x = sum x^2 - (sum x)^2 / n.
__global__ void unary_pearson_kernel(const double* __restrict__ colstats,
                                     const double* __restrict__ ystats, int64_t f,
                                     double* __restrict__ out) {
    int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= f) return;
    double n = ystats[0], var_y = ystats[2];
    double sx = colstats[c * 4], sxx = colstats[c * 4 + 1], dot = colstats[c * 4 + 2];
    double r = 0.0;
    if (n > 0.0) {
        double var_x = sxx - sx * (sx / n);
        if (var_x > 0.0 && var_y > 0.0) r = dot / sqrt(var_x * var_y);
    }
    out[c] = r;
}

}  // namespace
}  // namespace gafime

extern "C" int gafime_unary_scores(ContiguousBucket bucket, int metric, int mi_bins,
                                   double* out_scores) {
    if (!bucket || !out_scores) return GAFIME_ERROR_INVALID_ARGS;
    if (metric != GAFIME_METRIC_PEARSON && metric != GAFIME_METRIC_MUTUAL_INFO) return GAFIME_ERROR_INVALID_ARGS;
    if (metric == GAFIME_METRIC_MUTUAL_INFO && (mi_bins < 2 || mi_bins > 255)) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    cudaSetDevice(b.device);
    ColumnStats cs;
    int st = prepare(b, 0, GAFIME_METRIC_PEARSON, cs, false);
    if (st != GAFIME_SUCCESS) return st;
    cudaError_t e = ensure(b.scores, (size_t)std::max<int64_t>(b.f, 1) * sizeof(double));
    if (e != cudaSuccess) return status_from(e);
    double* d_out = (double*)b.scores.ptr;
    if (metric == GAFIME_METRIC_PEARSON) {
        unary_pearson_kernel<<<(unsigned)((b.f + 127) / 128), 128, 0, b.stream>>>(cs.d_col, cs.d_y, b.f, d_out);
        e = cudaGetLastError();
    } else {
        e = launch_mi_unary(b, mi_bins, d_out, b.stream);
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_scores, d_out, (size_t)b.f * sizeof(double), cudaMemcpyDeviceToHost, b.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    return status_from(e);
}

extern "C" int gafime_shard_tiles(int n_features, int shard_id, int n_shards, int32_t* out_tiles,
                                  int max_tiles, int* out_count) {
    if (n_features < 0 || n_shards < 1 || shard_id < 0 || shard_id >= n_shards || !out_count ||
        max_tiles < 0 || (max_tiles > 0 && !out_tiles))
        return GAFIME_ERROR_INVALID_ARGS;
    std::vector<TileCoord> t = gafime::shard_tiles(n_features, shard_id, n_shards);
    *out_count = (int)t.size();
    if ((int)t.size() > max_tiles) return GAFIME_ERROR_INVALID_ARGS;
    for (size_t q = 0; q < t.size(); ++q) {
        out_tiles[2 * q] = t[q].bi;
        out_tiles[2 * q + 1] = t[q].bj;
    }
    return GAFIME_SUCCESS;
}

// ---- streamed ingest: the host copy overlapped with scoring -------------------------------

namespace gafime {
namespace {

// 128-column block whose arrival completes a 64-tile (the later of its two blocks)
int arrival_block(const TileCoord& t) { return std::max(t.bi, t.bj) / 2; }

cudaError_t ensure_copy_stream(Bucket& b, size_t n_events) {
    cudaError_t e = cudaSuccess;
    if (!b.copy_stream) e = cudaStreamCreateWithFlags(&b.copy_stream, cudaStreamNonBlocking);
    while (e == cudaSuccess && b.arrived.size() < n_events) {
        cudaEvent_t ev;
        e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        if (e == cudaSuccess) b.arrived.push_back(ev);
    }
    return e;
}

// Upload + top-k with the copy of column block J overlapped with the scoring of the tiles
// that block J completes.  Same results as gafime_contiguous_bucket_upload followed by
// gafime_allpairs_topk (the per-column statistics and every tile's moments are computed by
// the same kernels on the same data; only the launch order differs).
int streamed_topk_body(Bucket& b, const float* h_data, const uint8_t* h_mask, const int* ops, int n_ops,
                       float div_eps, int k, int shard_id, int n_shards, int32_t* out_i, int32_t* out_j,
                       double* out_score, int* out_count) {
    const int64_t f = b.f, n = b.n, ld = b.ld;
    constexpr int64_t kBlock = 2 * kTile;  // the 128-column block of the tensor-core Gram tile
    const int nb = (int)((f + kBlock - 1) / kBlock);
    cudaError_t e = ensure_copy_stream(b, (size_t)nb + 1);
    if (e != cudaSuccess) return status_from(e);
    // tiles of this shard ordered by the block that completes them
    Plan plan = make_plan(b, shard_id, n_shards);
    std::stable_sort(plan.tiles.begin(), plan.tiles.end(),
                     [](const TileCoord& x, const TileCoord& z) { return arrival_block(x) < arrival_block(z); });
    const int nt = (int)plan.tiles.size();
    // the column blocks this shard's tiles read are the ones copied (all of them for one
    // shard, or when the shard has no tile and the call is a plain upload)
    std::vector<char> used((size_t)nb, nt == 0 ? 1 : 0);
    for (const TileCoord& t : plan.tiles) used[(size_t)(t.bi / 2)] = used[(size_t)(t.bj / 2)] = 1;
    bool all_blocks = true;
    for (int J = 0; J < nb; ++J) all_blocks = all_blocks && used[(size_t)J];
    // the target and the fold mask first, then the column blocks in order
    float* y = b.d_data + f * ld;
    e = cudaMemcpyAsync(y, h_data + f * n, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, b.copy_stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b.d_mask, h_mask, (size_t)n, cudaMemcpyHostToDevice, b.copy_stream);
    if (e == cudaSuccess) e = cudaEventRecord(b.arrived[(size_t)nb], b.copy_stream);
    for (int J = 0; J < nb && e == cudaSuccess; ++J) {
        if (!used[(size_t)J]) continue;
        const int64_t c0 = (int64_t)J * kBlock, c1 = std::min<int64_t>(f, c0 + kBlock);
        e = cudaMemcpy2DAsync(b.d_data + c0 * ld, (size_t)ld * sizeof(float), h_data + c0 * n,
                              (size_t)n * sizeof(float), (size_t)n * sizeof(float), (size_t)(c1 - c0),
                              cudaMemcpyHostToDevice, b.copy_stream);
        if (e == cudaSuccess) e = cudaEventRecord(b.arrived[(size_t)J], b.copy_stream);
    }
    if (e != cudaSuccess) return status_from(e);
    b.finite_state = -1;
    if (nt == 0) {
        // nothing to score on this shard: the upload alone, checked as an upload is
        e = cudaStreamSynchronize(b.copy_stream);
        if (e != cudaSuccess) return status_from(e);
        bool finite = true;
        return check_finite(b, &finite);
    }
    // the row chunks of the matrix and the Gram kernel the whole tile set would get (same
    // partial sums as an unstreamed call)
    const int64_t chunk = gram_chunk_rows(b);
    const int planes = gram_use_planes(b, plan.tiles) ? 1 : 0;
    TileCoord* d_tiles = nullptr;
    int st = upload_tiles(b, plan, &d_tiles);
    if (st != GAFIME_SUCCESS) return st;
    e = ensure(b.flags, 64);
    if (e != cudaSuccess) return status_from(e);
    int* flag = (int*)b.flags.ptr;
    e = cudaMemsetAsync(flag, 0, sizeof(int), b.stream);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(b.stream, b.arrived[(size_t)nb], 0);
    if (e == cudaSuccess) e = launch_finite_check(y, ld, flag, b.sm_count, b.stream);
    if (e != cudaSuccess) return status_from(e);
    ColumnStats cs;
    {
        KernelTimer timer(b.stream, GAFIME_KERNEL_COLUMN_STATS);
        st = compute_column_stats(b, false, cs, false);  // the target's statistics; columns below
    }
    if (st != GAFIME_SUCCESS) return st;
    e = gram_prep_target(b, cs, b.stream);
    if (e != cudaSuccess) return status_from(e);

    bool need[2] = {false, false};
    for (int o = 0; o < n_ops; ++o) need[ops[o] == GAFIME_INTERACT_DIV ? 1 : 0] = true;
    const size_t per_tile = (size_t)3 * kTilePairs;
    e = ensure(b.moments, 2 * std::max(1, nt) * per_tile * sizeof(double));
    if (e != cudaSuccess) return status_from(e);
    double* mom[2] = {(double*)b.moments.ptr, (double*)b.moments.ptr + std::max(1, nt) * per_tile};
    e = gram_error_reset(b, b.stream);
    if (e != cudaSuccess) return status_from(e);
    int t0 = 0;
    for (int J = 0; J < nb; ++J) {
        if (!used[(size_t)J]) continue;  // no tile of this shard reads it: not copied
        const int64_t c0 = (int64_t)J * kBlock, c1 = std::min<int64_t>(f, c0 + kBlock);
        e = cudaStreamWaitEvent(b.stream, b.arrived[(size_t)J], 0);
        if (e == cudaSuccess) e = launch_finite_check(b.d_data + c0 * ld, (c1 - c0) * ld, flag, b.sm_count, b.stream);
        if (e == cudaSuccess) e = gram_prep_columns(b, cs, need[1], div_eps, c0, c1, b.stream);
        if (e != cudaSuccess) return status_from(e);
        int t1 = t0;
        while (t1 < nt && arrival_block(plan.tiles[(size_t)t1]) == J) ++t1;
        if (t1 == t0) continue;
        const std::vector<TileCoord> sub(plan.tiles.begin() + t0, plan.tiles.begin() + t1);
        for (int g2 = 0; g2 < 2; ++g2) {
            if (!need[g2]) continue;
            e = launch_gram_moments(b, cs, d_tiles + t0, sub, g2 == 1, div_eps, mom[g2] + (size_t)t0 * per_tile,
                                    b.stream, nullptr, GRAM_PREP_DONE, chunk, planes);
            if (e != cudaSuccess) return status_from(e);
        }
        t0 = t1;
    }
    e = cudaStreamSynchronize(b.copy_stream);
    if (e != cudaSuccess) return status_from(e);

    const int k_pad = next_pow2(k);
    const int sub_lists = epilogue_sub_lists(nt, k_pad, b.sm_count);
    const int n_lists = nt * sub_lists;
    const size_t per_op = (size_t)n_lists * k_pad;
    e = ensure(b.cands, per_op * n_ops * sizeof(Cand));
    if (e == cudaSuccess) e = ensure(b.cands2, per_op * n_ops * sizeof(Cand));
    if (e != cudaSuccess) return status_from(e);
    Cand* cands[4];
    Cand* tmp[4];
    for (int o = 0; o < n_ops; ++o) {
        cands[o] = (Cand*)b.cands.ptr + per_op * o;
        tmp[o] = (Cand*)b.cands2.ptr + per_op * o;
    }
    st = queue_epilogue(b, cs, d_tiles, nt, ops, n_ops, mom[0], 1, mom[1], 1, k_pad, sub_lists, cands, nullptr,
                        div_eps, true);
    if (st != GAFIME_SUCCESS) return st;
    st = merge_and_copy(b, cands, tmp, n_lists, k, k_pad, n_ops, per_op, out_i, out_j, out_score, out_count);
    if (st == GAFIME_SUCCESS) st = gram_status(b, 1);
    if (st != GAFIME_SUCCESS) {
        for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
        return st;
    }
    // the ingest check of an upload: results over non-finite data are discarded
    int h = 0;
    e = cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, b.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return status_from(e);
    // a shard that copied part of the matrix leaves the rest unchecked for later calls
    b.finite_state = h != 0 ? 0 : (all_blocks ? 1 : -1);
    if (h != 0) {
        for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
        return GAFIME_ERROR_INVALID_ARGS;
    }
    return GAFIME_SUCCESS;
}

// streamed_topk_body, and on a failed call the copy stream drained before returning: the
// caller may free or refill its host buffers as soon as the call returns
int streamed_topk(Bucket& b, const float* h_data, const uint8_t* h_mask, const int* ops, int n_ops, float div_eps,
                  int k, int shard_id, int n_shards, int32_t* out_i, int32_t* out_j, double* out_score,
                  int* out_count) {
    const int st = streamed_topk_body(b, h_data, h_mask, ops, n_ops, div_eps, k, shard_id, n_shards, out_i, out_j,
                                      out_score, out_count);
    if (st != GAFIME_SUCCESS && b.copy_stream) cudaStreamSynchronize(b.copy_stream);
    return st;
}

}  // namespace
}  // namespace gafime

extern "C" int gafime_allpairs_topk_host(ContiguousBucket bucket, const float* h_data, const uint8_t* h_mask,
                                         const int* interact_types, int n_ops, int metric, int center,
                                         float div_eps, int mi_bins, int k, int shard_id, int n_shards,
                                         int32_t* out_i, int32_t* out_j, double* out_score, int* out_count) {
    if (!bucket || !h_data || !h_mask || !interact_types || n_ops < 1 || n_ops > 4 || k < 1 ||
        k > GAFIME_ALLPAIRS_MAX_K || n_shards < 1 || shard_id < 0 || shard_id >= n_shards || !out_i || !out_j ||
        !out_score || !out_count)
        return GAFIME_ERROR_INVALID_ARGS;
    if (!valid_metric(metric)) return GAFIME_ERROR_INVALID_ARGS;
    if (metric != GAFIME_METRIC_PEARSON && (mi_bins < 2 || mi_bins > 255)) return GAFIME_ERROR_INVALID_ARGS;
    if (!(div_eps > 0.0f)) return GAFIME_ERROR_INVALID_ARGS;
    for (int o = 0; o < n_ops; ++o)
        if (!valid_op(interact_types[o])) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    if (b.f >= 65536) return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(b.device);
    b.last_rescored = 0;
    b.guard_ran = false;
    for (int o = 0; o < n_ops; ++o) out_count[o] = 0;
    // the tensor-core Pearson path streams; the others score after a plain upload
    if (metric == GAFIME_METRIC_PEARSON && center == 0 && gram_path_enabled(b) && b.f >= 2)
        return streamed_topk(b, h_data, h_mask, interact_types, n_ops, div_eps, k, shard_id, n_shards, out_i,
                             out_j, out_score, out_count);
    int st = gafime_contiguous_bucket_upload(bucket, h_data, h_mask);
    if (st != GAFIME_SUCCESS) return st;
    return gafime_allpairs_topk(bucket, interact_types, n_ops, metric, center, div_eps, mi_bins, k, shard_id,
                                n_shards, out_i, out_j, out_score, out_count);
}

extern "C" int gafime_allpairs_rescored(ContiguousBucket bucket, int64_t* out_count) {
    if (!bucket || !out_count) return GAFIME_ERROR_INVALID_ARGS;
    *out_count = ((Bucket*)bucket)->last_rescored;
    return GAFIME_SUCCESS;
}
