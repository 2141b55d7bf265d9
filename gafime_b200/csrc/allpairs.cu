// allpairs.cu -- host scheduler of the all-pairs scoring call.
//
// Replaces the reference's per-pair loop (gafime/backends/native_cuda_backend.py:368-379:
// one launch + memset + D2H + sync per pair) and its Rust pair enumeration
// (src/cpu/gafime_cpu/src/batch_launcher.rs:216-247, smart_scheduler.rs:78-176) with:
//   1. fp64 column statistics (bucket.cu), once per call;
//   2. upper-triangle 64 x 64 pair tiles, assigned to shards by pair count;
//   3. split-K over rows so every SM has work, fp64 partials per (tile, split);
//   4. the scoring epilogue with a per-tile bitonic top-k, one launch per operator;
//   5. a device merge of the per-tile lists and one small D2H per operator.
// Everything is queued on the bucket's stream; the only host sync is the final copy.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
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
// 128 x 128 blocks (the tensor-core Gram tile): blocks in decreasing pair count (ties in
// row-major order), each to the shard with the fewest pairs so far (ties: lowest shard
// id); a shard scores the 64-tiles inside its blocks.  Every process derives the same
// split without communication.
std::vector<TileCoord> shard_tiles(int64_t f, int shard_id, int n_shards) {
    int nb = (int)((f + kTile - 1) / kTile);
    int nb2 = (nb + 1) / 2;
    struct Block {
        int64_t w;
        int order, ns;
        TileCoord sub[4];
    };
    std::vector<Block> blocks;
    for (int BI = 0; BI < nb2; ++BI)
        for (int BJ = BI; BJ < nb2; ++BJ) {
            Block blk{0, (int)blocks.size(), 0, {}};
            for (int da = 0; da < 2; ++da)
                for (int db = 0; db < 2; ++db) {
                    int bi = 2 * BI + da, bj = 2 * BJ + db;
                    if (bi > bj || bi >= nb || bj >= nb) continue;
                    int64_t p = tile_pairs(bi, bj, f);
                    if (p == 0) continue;
                    blk.sub[blk.ns++] = {bi, bj};
                    blk.w += p;
                }
            if (blk.w > 0) blocks.push_back(blk);
        }
    std::stable_sort(blocks.begin(), blocks.end(),
                     [](const Block& x, const Block& y) { return x.w > y.w; });
    std::vector<int64_t> load((size_t)n_shards, 0);
    std::vector<TileCoord> mine;
    for (const Block& blk : blocks) {
        int best = 0;
        for (int s = 1; s < n_shards; ++s)
            if (load[(size_t)s] < load[(size_t)best]) best = s;
        load[(size_t)best] += blk.w;
        if (best == shard_id)
            for (int q = 0; q < blk.ns; ++q) mine.push_back(blk.sub[q]);
    }
    return mine;
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
    int nt = (int)p.tiles.size();
    int splits = nt > 0 ? std::max(1, b.sm_count / nt) : 1;
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

// Queue moments + epilogue for the requested operators.  cands[o] receives n_tiles *
// sub_lists lists of k_pad entries for operator o (nullptr: no selection); mutual
// information writes n_tiles lists.
int score_ops(Bucket& b, const ColumnStats& cs, const Plan& plan, const TileCoord* d_tiles,
              const int* ops, int n_ops, int metric, int center, float div_eps, int mi_bins,
              int k_pad, int sub_lists, Cand* const* cands, double* all_scores) {
    const int nt = (int)plan.tiles.size();
    if (nt == 0) return GAFIME_SUCCESS;
    cudaError_t e;
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
    for (int g = 0; g < 2; ++g) {
        if (!need[g]) continue;
        if (tensor) {
            int gerr = 0;
            // one operand preparation serves both groups when both are scored
            const int prep = (g == 0 && need[1]) ? GRAM_PREP_BOTH : (g == 1 && need[0]) ? GRAM_PREP_DONE
                                                                                      : GRAM_PREP_OWN;
            e = launch_gram_moments(b, cs, d_tiles, plan.tiles, g == 1, div_eps, mom[g], b.stream, &gerr,
                                    prep);
            if (e != cudaSuccess) return status_from(e);
            if (gerr) return GAFIME_ERROR_KERNEL_FAILED;
            group_splits[g] = 1;
        } else {
            KernelTimer timer(b.stream, GAFIME_KERNEL_PAIR_MOMENTS);
            e = launch_pair_moments(cs.d_x, b.ld, cs.d_ycen, b.f, d_tiles, nt, plan.splits,
                                    plan.rows_per_split, g == 1, div_eps, mom[g], b.stream);
            if (e != cudaSuccess) return status_from(e);
        }
    }
    EpilogueArgs a;
    for (int o = 0; o < n_ops; ++o) {
        const int grp = ops[o] == GAFIME_INTERACT_DIV ? 1 : 0;
        a.moments[o] = mom[grp];
        a.splits[o] = group_splits[grp];
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
    {
        KernelTimer timer(b.stream, GAFIME_KERNEL_EPILOGUE_TOPK);
        e = launch_epilogue_topk(a, b.stream);
    }
    if (e != cudaSuccess) return status_from(e);
    return GAFIME_SUCCESS;
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

extern "C" int gafime_allpairs_topk(ContiguousBucket bucket, const int* interact_types, int n_ops,
                                    int metric, int center, float div_eps, int mi_bins, int k,
                                    int shard_id, int n_shards, int32_t* out_i, int32_t* out_j,
                                    double* out_score, int* out_count) {
    if (!bucket || !interact_types || n_ops < 1 || n_ops > 4 || k < 1 || k > GAFIME_ALLPAIRS_MAX_K ||
        n_shards < 1 || shard_id < 0 || shard_id >= n_shards || !out_i || !out_j || !out_score ||
        !out_count)
        return GAFIME_ERROR_INVALID_ARGS;
    if (metric != GAFIME_METRIC_PEARSON && metric != GAFIME_METRIC_MUTUAL_INFO) return GAFIME_ERROR_INVALID_ARGS;
    if (metric == GAFIME_METRIC_MUTUAL_INFO && (mi_bins < 2 || mi_bins > 255)) return GAFIME_ERROR_INVALID_ARGS;
    if (!(div_eps > 0.0f)) return GAFIME_ERROR_INVALID_ARGS;
    for (int o = 0; o < n_ops; ++o)
        if (!valid_op(interact_types[o])) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    if (b.f >= 65536) return GAFIME_ERROR_INVALID_ARGS;  // pair id i*F + j must fit 32 bits
    cudaSetDevice(b.device);
    for (int o = 0; o < n_ops; ++o) out_count[o] = 0;

    Plan plan = make_plan(b, shard_id, n_shards);
    const int nt = (int)plan.tiles.size();
    if (nt == 0) return GAFIME_SUCCESS;
    ColumnStats cs;
    int st = prepare(b, center, metric, cs, true);
    if (st != GAFIME_SUCCESS) return st;
    TileCoord* d_tiles = nullptr;
    st = upload_tiles(b, plan, &d_tiles);
    if (st != GAFIME_SUCCESS) return st;

    const int k_pad = next_pow2(k);
    const int sub_lists = metric == GAFIME_METRIC_PEARSON ? epilogue_sub_lists(nt, k_pad, b.sm_count) : 1;
    const int n_lists = nt * sub_lists;
    size_t per_op = (size_t)n_lists * k_pad;
    cudaError_t e = ensure(b.cands, per_op * n_ops * sizeof(Cand));
    if (e == cudaSuccess) e = ensure(b.cands2, per_op * n_ops * sizeof(Cand));
    if (e != cudaSuccess) return status_from(e);
    Cand* cands[4];
    Cand* tmp[4];
    for (int o = 0; o < n_ops; ++o) {
        cands[o] = (Cand*)b.cands.ptr + per_op * o;
        tmp[o] = (Cand*)b.cands2.ptr + per_op * o;
    }
    st = score_ops(b, cs, plan, d_tiles, interact_types, n_ops, metric, center, div_eps, mi_bins,
                   k_pad, sub_lists, cands, nullptr);
    if (st != GAFIME_SUCCESS) return st;

    std::vector<Cand> host((size_t)k_pad * n_ops);
    Cand* fin = nullptr;
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
    e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return status_from(e);
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

extern "C" int gafime_allpairs_scores(ContiguousBucket bucket, int interact_type, int metric,
                                      int center, float div_eps, int mi_bins, double* out_scores) {
    if (!bucket || !out_scores || !valid_op(interact_type)) return GAFIME_ERROR_INVALID_ARGS;
    if (metric != GAFIME_METRIC_PEARSON && metric != GAFIME_METRIC_MUTUAL_INFO) return GAFIME_ERROR_INVALID_ARGS;
    if (metric == GAFIME_METRIC_MUTUAL_INFO && (mi_bins < 2 || mi_bins > 255)) return GAFIME_ERROR_INVALID_ARGS;
    if (!(div_eps > 0.0f)) return GAFIME_ERROR_INVALID_ARGS;
    Bucket& b = *(Bucket*)bucket;
    if (b.f >= 65536) return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(b.device);
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
    st = score_ops(b, cs, plan, d_tiles, &interact_type, 1, metric, center, div_eps, mi_bins, 1, 1,
                   none, (double*)b.scores.ptr);
    if (st != GAFIME_SUCCESS) return st;
    e = cudaMemcpyAsync(out_scores, b.scores.ptr, (size_t)P * sizeof(double), cudaMemcpyDeviceToHost,
                        b.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    return status_from(e);
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
