// select.cu -- scoring epilogue fused with a block-level bitonic top-k, the
// device merge of per-tile candidate lists, and the host merge across shards.
//
// Pearson from the moments (per pair, fp64), following the reference's
// _pearson_from_stats (native_cuda_backend.py:471-486) and gafime_core's
// pearson_from_sums (gafime_core.cpp:179-198):
//     r = cov / sqrt(var_x * var_y),   r = 0 when n <= 1 or var_x*var_y <= 0
// with, per operator (a = X[:, i], b = X[:, j], i < j; S* from moments.cu, per-column
// sums Sa = sum a, Qa = sum a^2, Ua = sum a*ycen):
//     multiply / divide : sum x = S1, sum x^2 = S2, cov = S3
//     add               : sum x = Sa + Sb, sum x^2 = Qa + 2 S1 + Qb, cov = Ua + Ub
//     subtract          : sum x = Sa - Sb, sum x^2 = Qa - 2 S1 + Qb, cov = Ua - Ub
//     var_x = sum x^2 - (sum x)^2 / n
// (cov uses ycen = y - mean y, so it equals sum xy - sum x sum y / n.)
// Ranking: |score| descending, then pair id i*F + j ascending (the reference
// sorts by abs(metric), gafime/sklearn.py:62-71; ties are ordered by pair).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "engine.h"
#include "select.cuh"

namespace gafime {

namespace {

constexpr int kEpiThreads = 256;

__device__ __forceinline__ double pearson(double n, double sx, double sxx, double cov, double var_y) {
    if (n <= 1.0) return 0.0;
    double var_x = sxx - sx * sx / n;
    double d = var_x * var_y;
    if (!(d > 0.0)) return 0.0;
    return cov / sqrt(d);
}

// Grid (n_tiles, sub_lists, n_ops): CTA (t, s, o) scores operator o on the pairs e in
// [s*L, (s+1)*L) of tile t (L = kTilePairs / sub_lists) and writes the k_pad best of them,
// sorted, as list t * sub_lists + s of that operator.
__global__ void __launch_bounds__(kEpiThreads) epilogue_topk_kernel(EpilogueArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Cand* s = reinterpret_cast<Cand*>(smem_raw);  // [L]
    const int t = blockIdx.x;
    const int oi = blockIdx.z;
    const int op = a.op[oi], splits = a.splits[oi];
    const double* moments = a.moments[oi];
    Cand* cands = a.cands[oi];
    const int L = kTilePairs / a.sub_lists;
    const int e0 = blockIdx.y * L;
    const TileCoord tc = a.tiles[t];
    const double n = a.ystats[0], var_y = a.ystats[2];
    const int64_t f = a.f;
    for (int q = threadIdx.x; q < L; q += kEpiThreads) {
        const int e = e0 + q;
        int li = e / kTile, lj = e % kTile;
        int64_t i = (int64_t)tc.bi * kTile + li, j = (int64_t)tc.bj * kTile + lj;
        Cand c;
        c.pad = 0;
        if (i < j && j < f) {
            double S1 = 0.0, S2 = 0.0, S3 = 0.0;
            for (int sp = 0; sp < splits; ++sp) {
                const double* m = moments + ((int64_t)sp * a.n_tiles + t) * 3 * kTilePairs;
                S1 += m[e];
                S2 += m[kTilePairs + e];
                S3 += m[2 * kTilePairs + e];
            }
            double sx, sxx, cov;
            if (op == GAFIME_INTERACT_ADD || op == GAFIME_INTERACT_SUB) {
                double sg = op == GAFIME_INTERACT_ADD ? 1.0 : -1.0;
                const double* ci = a.colstats + i * 4;
                const double* cj = a.colstats + j * 4;
                sx = ci[0] + sg * cj[0];
                sxx = ci[1] + 2.0 * sg * S1 + cj[1];
                cov = ci[2] + sg * cj[2];
            } else {
                sx = S1;
                sxx = S2;
                cov = S3;
            }
            c.score = pearson(n, sx, sxx, cov, var_y);
            if (a.guard_flags) {
                // a pair the accuracy guard flagged takes its exact re-score (guard.cu)
                const int64_t g = ((int64_t)oi * a.n_tiles + t) * kTilePairs + e;
                if (a.guard_flags[g]) c.score = a.exact[g];
            }
            c.pid = (uint32_t)(i * f + j);
            if (a.all_scores) {
                int64_t p = i * f - i * (i + 1) / 2 + (j - i - 1);
                a.all_scores[p] = c.score;
            }
        } else {
            c.score = 0.0;
            c.pid = kNoPair;
        }
        s[q] = c;
    }
    if (cands == nullptr) return;  // scores only (uniform across the block)
    __syncthreads();
    bitonic_sort(s, L);
    Cand* out = cands + ((int64_t)t * a.sub_lists + blockIdx.y) * a.k_pad;
    for (int q = threadIdx.x; q < a.k_pad; q += kEpiThreads) out[q] = s[q];
}

// Each CTA reduces `group` consecutive sorted lists (k_pad entries each; lists beyond
// n_lists are empty) of operator blockIdx.y to their k_pad best entries, sorted.  Pairwise tree: for runs A and B
// sorted best-first, better(A[i], B[k-1-i]) over i is a bitonic sequence holding the k best
// of A and B, which log2(k) half-cleaner stages sort.
__global__ void __launch_bounds__(1024) merge_kernel(const Cand* __restrict__ in, int n_lists,
                                                     int k_pad, int group, int64_t op_stride,
                                                     Cand* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Cand* s = reinterpret_cast<Cand*>(smem_raw);
    const int g = blockIdx.x;
    in += blockIdx.y * op_stride;
    out += blockIdx.y * op_stride;
    const int total = group * k_pad;
    for (int e = threadIdx.x; e < total; e += blockDim.x) {
        int l = g * group + e / k_pad;
        if (l < n_lists) {
            s[e] = in[(int64_t)l * k_pad + (e % k_pad)];
        } else {
            Cand c;
            c.score = 0.0;
            c.pid = kNoPair;
            c.pad = 0;
            s[e] = c;
        }
    }
    __syncthreads();
    for (int span = 1; span < group; span <<= 1) {
        // runs a = 2*span*q keep the k best of runs a and a + span
        const int pairs = group / (2 * span);
        for (int e = threadIdx.x; e < pairs * k_pad; e += blockDim.x) {
            const int q = e / k_pad, i = e % k_pad;
            const int ra = 2 * span * q;
            Cand* A = s + (int64_t)ra * k_pad;
            const Cand& bv = s[(int64_t)(ra + span) * k_pad + (k_pad - 1 - i)];
            if (cand_before(bv, A[i])) A[i] = bv;
        }
        __syncthreads();
        for (int stride = k_pad >> 1; stride > 0; stride >>= 1) {
            for (int e = threadIdx.x; e < pairs * (k_pad >> 1); e += blockDim.x) {
                const int q = e / (k_pad >> 1), r = e % (k_pad >> 1);
                Cand* A = s + (int64_t)(2 * span * q) * k_pad;
                const int i = 2 * stride * (r / stride) + (r % stride);
                cand_cswap(A, i, i + stride, true);
            }
            __syncthreads();
        }
    }
    for (int e = threadIdx.x; e < k_pad; e += blockDim.x) out[(int64_t)g * k_pad + e] = s[e];
}

__global__ void fill_empty_kernel(Cand* out, size_t n) {
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        Cand c;
        c.score = 0.0;
        c.pid = kNoPair;
        c.pad = 0;
        out[e] = c;
    }
}

__global__ void reorder_kernel(const Cand* __restrict__ in, Cand* __restrict__ out, int n_shards, int n_ops,
                               int k_pad) {
    const size_t total = (size_t)n_shards * n_ops * k_pad;
    for (size_t x = (size_t)blockIdx.x * blockDim.x + threadIdx.x; x < total; x += (size_t)gridDim.x * blockDim.x) {
        const size_t s = x / ((size_t)n_ops * k_pad), o = (x / k_pad) % n_ops, e = x % k_pad;
        out[(o * n_shards + s) * k_pad + e] = in[x];
    }
}

}  // namespace

cudaError_t fill_empty_lists(Cand* out, size_t n, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    fill_empty_kernel<<<(unsigned)std::min<size_t>(1024, (n + 255) / 256), 256, 0, stream>>>(out, n);
    return cudaGetLastError();
}

cudaError_t reorder_shard_lists(const Cand* in, Cand* out, int n_shards, int n_ops, int k_pad, cudaStream_t stream) {
    const size_t total = (size_t)n_shards * n_ops * k_pad;
    reorder_kernel<<<(unsigned)std::min<size_t>(1024, (total + 255) / 256), 256, 0, stream>>>(in, out, n_shards, n_ops,
                                                                                           k_pad);
    return cudaGetLastError();
}

cudaError_t launch_epilogue_topk(const EpilogueArgs& a, cudaStream_t stream) {
    if (a.n_tiles <= 0) return cudaSuccess;
    if (a.n_ops < 1 || a.n_ops > 4 || a.sub_lists < 1 || kTilePairs % a.sub_lists != 0) return cudaErrorInvalidValue;
    for (int o = 0; o < a.n_ops; ++o)
        if (a.cands[o] && kTilePairs / a.sub_lists < a.k_pad) return cudaErrorInvalidValue;
    size_t smem = sizeof(Cand) * (kTilePairs / a.sub_lists);
    cudaFuncSetAttribute(epilogue_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    epilogue_topk_kernel<<<dim3((unsigned)a.n_tiles, (unsigned)a.sub_lists, (unsigned)a.n_ops), kEpiThreads, smem,
                           stream>>>(a);
    return cudaGetLastError();
}

int epilogue_sub_lists(int n_tiles, int k_pad, int sm_count) {
    // More lists per tile give the epilogue more CTAs; few enough lists that one merge CTA
    // (8192 entries) can take them all keep the merge to one launch.  Each list stays at
    // least k_pad long.
    const int64_t cap = std::min<int64_t>(2 * (int64_t)sm_count, std::max<int64_t>(n_tiles, 8192 / k_pad));
    int s = 1;
    while (2 * s <= kTilePairs / k_pad && (int64_t)n_tiles * 2 * s <= cap) s <<= 1;
    return s;
}

cudaError_t merge_candidates(Cand* buf, Cand* tmp, int n_lists, int k_pad, int n_ops, size_t op_stride,
                             Cand** final_list, cudaStream_t stream) {
    // lists per CTA: a power of two, group * k_pad <= 8192 entries (128 KB of shared memory),
    // no more than the lists there are
    int fit = std::max(2, 8192 / k_pad);
    int group = 2;
    while (group < fit && group < n_lists) group <<= 1;
    size_t smem = sizeof(Cand) * (size_t)group * k_pad;
    cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    Cand* src = buf;
    Cand* dst = tmp;
    while (n_lists > 1) {
        int out_lists = (n_lists + group - 1) / group;
        merge_kernel<<<dim3((unsigned)out_lists, (unsigned)n_ops), 1024, smem, stream>>>(src, n_lists, k_pad, group,
                                                                                    (int64_t)op_stride, dst);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        std::swap(src, dst);
        n_lists = out_lists;
    }
    *final_list = src;
    return cudaSuccess;
}

}  // namespace gafime

using namespace gafime;

extern "C" int gafime_topk_merge(const int32_t* cand_i, const int32_t* cand_j,
                                 const double* cand_score, int64_t n_cand, int k, int32_t* out_i,
                                 int32_t* out_j, double* out_score, int* out_count) {
    if (n_cand < 0 || k <= 0 || !out_i || !out_j || !out_score || !out_count) return GAFIME_ERROR_INVALID_ARGS;
    if (n_cand > 0 && (!cand_i || !cand_j || !cand_score)) return GAFIME_ERROR_INVALID_ARGS;
    struct E {
        double s;
        int32_t i, j;
    };
    std::vector<E> v;
    v.reserve((size_t)n_cand);
    for (int64_t c = 0; c < n_cand; ++c) {
        if (cand_i[c] < 0 || cand_j[c] < 0) continue;  // empty slots
        int32_t lo = std::min(cand_i[c], cand_j[c]), hi = std::max(cand_i[c], cand_j[c]);
        v.push_back({cand_score[c], lo, hi});
    }
    auto rank = [](double s) { return s != s ? -1.0 : (s < 0 ? -s : s); };
    std::sort(v.begin(), v.end(), [&](const E& a, const E& b) {
        double ra = rank(a.s), rb = rank(b.s);
        if (ra != rb) return ra > rb;
        if (a.i != b.i) return a.i < b.i;
        return a.j < b.j;
    });
    int m = (int)std::min<int64_t>((int64_t)k, (int64_t)v.size());
    for (int c = 0; c < m; ++c) {
        out_i[c] = v[c].i;
        out_j[c] = v[c].j;
        out_score[c] = v[c].s;
    }
    *out_count = m;
    return GAFIME_SUCCESS;
}
