// rank.cu -- Spearman rank correlation of interactions against the target.
//
// Semantics of gafime_core.score_combos for the "spearman" metric
// (gafime_core.cpp:595-607):
//   ranks   : rankdata (gafime_core.cpp:156-177): stable order of the values, a run of equal
//             values shares the average 0-based rank 0.5 * (first + last);
//   target  : y ranks centred by their mean, var = sum r^2 - sum r * mean
//             (gafime_core.cpp:503-517);
//   score   : pearson_from_sums(sum r, sum r^2, sum r * ycen_rank, var_y_rank, n)
//             (gafime_core.cpp:179-198).
//   x       : a one-feature combo is the raw column (gafime_core.cpp:558-568); a pair is
//             (a - mean_a) op (b - mean_b) in fp64 (center = 1; for multiply the reference's
//             centred product, gafime_core.cpp:571-577) or fl32(a op b) (center = 0, the
//             kernel-API interaction, cpu_backend.cpp:87-103).
//
// Device plan per combo: order-preserving integer keys of x (32-bit for fp32 values, 64-bit
// for fp64 products; -0.0 keyed as +0.0 so the two compare equal as in the reference) and row
// ids are radix-sorted (CUB, device-wide); run heads are flagged, a max-scan gives every
// position its run's first index, each run's end is written at its first index, and one
// fused pass forms the average rank and the three fp64 sums (per-block partials, then a
// fixed-order final sum: deterministic).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "engine.h"

namespace gafime {

namespace {

constexpr int kRankBlocks = 296;  // 2 x 148 SMs; fixed so the partial-sum order is fixed
constexpr int kRankThreads = 256;

__device__ __forceinline__ uint32_t okey(float v) {
    v = v + 0.0f;  // -0.0 -> +0.0
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ uint64_t okey(double v) {
    v = v + 0.0;
    const uint64_t b = (uint64_t)__double_as_longlong(v);
    return (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);
}

template <typename T>
__device__ __forceinline__ T combine(T a, T b, int op, T eps) {
    switch (op) {
        case GAFIME_INTERACT_ADD: return a + b;
        case GAFIME_INTERACT_SUB: return a - b;
        case GAFIME_INTERACT_DIV: return a / (fabs((double)b) < (double)eps ? (T)copysign((double)eps, (double)b) : b);
        default: return a * b;
    }
}

// keys and row ids of x for one combo.  kind: 0 raw column, 1 fl32(a op b), 2 fp64 centred
template <typename K>
__global__ void fill_keys_kernel(const float* __restrict__ x, int64_t ld, int64_t n, int a, int b, int kind,
                                 int op, float eps, double mean_a, double mean_b, K* __restrict__ keys,
                                 int32_t* __restrict__ ids) {
    const float* ca = x + (int64_t)a * ld;
    const float* cb = x + (int64_t)(b < 0 ? a : b) * ld;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
        if constexpr (sizeof(K) == 4) {
            const float v = kind == 0 ? ca[r] : combine<float>(ca[r], cb[r], op, eps);
            keys[r] = okey(v);
        } else {
            const double v = combine<double>((double)ca[r] - mean_a, (double)cb[r] - mean_b, op, (double)eps);
            keys[r] = okey(v);
        }
        ids[r] = (int32_t)r;
    }
}

// start[i] = i at a run head (first of equal keys in sorted order), else 0
template <typename K>
__global__ void heads_kernel(const K* __restrict__ keys, int64_t n, int32_t* __restrict__ start) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        start[i] = (i == 0 || keys[i] != keys[i - 1]) ? (int32_t)i : 0;
}

// after the max-scan start[i] is the first index of i's run; end_of[first] = one past its last
__global__ void run_ends_kernel(const int32_t* __restrict__ start, int64_t n, int32_t* __restrict__ end_of) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        if (i + 1 == n)
            end_of[start[i]] = (int32_t)n;
        else if (start[i + 1] == i + 1)
            end_of[start[i]] = (int32_t)(i + 1);
    }
}

__device__ __forceinline__ double avg_rank(const int32_t* start, const int32_t* end_of, int64_t i) {
    const int32_t s = start[i];
    return 0.5 * (double)((int64_t)s + (int64_t)end_of[s] - 1);
}

// Block partials of sum r, sum r^2 and sum r * ycr[id] (ycr null: no dot product); with
// rank_out set, rank_out[id] = r as well (the target's ranks in row order).
__global__ void __launch_bounds__(kRankThreads) rank_sums_kernel(const int32_t* __restrict__ start,
                                                                 const int32_t* __restrict__ end_of,
                                                                 const int32_t* __restrict__ ids, int64_t n,
                                                                 const double* __restrict__ ycr,
                                                                 double* __restrict__ rank_out,
                                                                 double* __restrict__ partial) {
    double s1 = 0.0, s2 = 0.0, s3 = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const double r = avg_rank(start, end_of, i);
        s1 += r;
        s2 += r * r;
        if (ycr) s3 += r * ycr[ids[i]];
        if (rank_out) rank_out[ids[i]] = r;
    }
    __shared__ double sh[3][kRankThreads];
    sh[0][threadIdx.x] = s1;
    sh[1][threadIdx.x] = s2;
    sh[2][threadIdx.x] = s3;
    __syncthreads();
    for (int w = kRankThreads / 2; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w)
            for (int q = 0; q < 3; ++q) sh[q][threadIdx.x] += sh[q][threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x < 3) partial[blockIdx.x * 3 + threadIdx.x] = sh[threadIdx.x][0];
}

__device__ __forceinline__ double pearson_from_sums(double sum_x, double sum_x2, double dot_xy, double var_y,
                                                    int64_t n) {
    if (n == 0) return 0.0;
    const double mean_x = sum_x / (double)n;
    const double var_x = sum_x2 - (sum_x * mean_x);
    if (var_x <= 0.0 || var_y <= 0.0) return 0.0;
    const double denom = sqrt(var_x * var_y);
    if (denom == 0.0) return 0.0;
    return dot_xy / denom;
}

// One thread: fixed-order sum of the block partials.  ystat = {mean_r, var_y_rank}.
// mode 0: the target (writes ystat); mode 1: a combo (writes its score to *out).
__global__ void rank_final_kernel(const double* __restrict__ partial, int blocks, int64_t n, int mode,
                                  double* __restrict__ ystat, double* __restrict__ out) {
    double s1 = 0.0, s2 = 0.0, s3 = 0.0;
    for (int b = 0; b < blocks; ++b) {
        s1 += partial[3 * b];
        s2 += partial[3 * b + 1];
        s3 += partial[3 * b + 2];
    }
    if (mode == 0) {
        const double mean_r = n == 0 ? 0.0 : s1 / (double)n;
        ystat[0] = mean_r;
        ystat[1] = s2 - (s1 * mean_r);
    } else {
        *out = pearson_from_sums(s1, s2, s3, ystat[1], n);
    }
}

__global__ void centre_kernel(const double* __restrict__ rank, int64_t n, const double* __restrict__ ystat,
                              double* __restrict__ ycr) {
    const double m = ystat[0];
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        ycr[r] = rank[r] - m;
}

struct RankScratch {
    void* keys[2];
    int32_t* ids[2];
    int32_t* start;
    int32_t* end_of;
    double* ycr;
    double* partial;
    double* ystat;
    void* temp;
    size_t temp_bytes;
};

struct MaxOp {
    __device__ __forceinline__ int32_t operator()(int32_t a, int32_t b) const { return a > b ? a : b; }
};

size_t cub_temp_bytes(int64_t n) {
    size_t a = 0, b = 0, c = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, a, (const uint64_t*)nullptr, (uint64_t*)nullptr, (const int32_t*)nullptr,
                                    (int32_t*)nullptr, (int)n);
    cub::DeviceRadixSort::SortPairs(nullptr, b, (const uint32_t*)nullptr, (uint32_t*)nullptr, (const int32_t*)nullptr,
                                    (int32_t*)nullptr, (int)n);
    cub::DeviceScan::InclusiveScan(nullptr, c, (const int32_t*)nullptr, (int32_t*)nullptr, MaxOp(), (int)n);
    return std::max(a, std::max(b, c));
}

// Sort (keys, ids) of scratch slot 0 into slot 1, then start / end_of of the sorted keys.
template <typename K>
cudaError_t sort_and_runs(RankScratch& s, int64_t n, int sm, cudaStream_t st) {
    size_t tb = s.temp_bytes;
    cudaError_t e = cub::DeviceRadixSort::SortPairs(s.temp, tb, (const K*)s.keys[0], (K*)s.keys[1],
                                                    (const int32_t*)s.ids[0], s.ids[1], (int)n, 0,
                                                    (int)(8 * sizeof(K)), st);
    if (e != cudaSuccess) return e;
    const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * sm));
    heads_kernel<K><<<g, 256, 0, st>>>((const K*)s.keys[1], n, s.start);
    tb = s.temp_bytes;
    e = cub::DeviceScan::InclusiveScan(s.temp, tb, s.start, s.start, MaxOp(), (int)n, st);
    if (e != cudaSuccess) return e;
    run_ends_kernel<<<g, 256, 0, st>>>(s.start, n, s.end_of);
    return cudaGetLastError();
}

}  // namespace

int spearman_scores(Bucket& b, const int32_t* feat_a, const int32_t* feat_b, int64_t n_combos, int op, int center,
                    float div_eps, double* out) {
    const int64_t n = b.n;
    cudaStream_t st = b.stream;
    // scratch: keys x2 (8 B), ids x2, start, end_of (4 B), ycr, y ranks (8 B), partials, ystat, scores, temp
    const size_t al = 256;
    auto up = [&](size_t v) { return (v + al - 1) / al * al; };
    const size_t tb = up(cub_temp_bytes(n));
    const size_t off_k0 = 0, off_k1 = off_k0 + up(8 * n), off_i0 = off_k1 + up(8 * n), off_i1 = off_i0 + up(4 * n);
    const size_t off_st = off_i1 + up(4 * n), off_en = off_st + up(4 * n), off_ycr = off_en + up(4 * n);
    const size_t off_yr = off_ycr + up(8 * n), off_part = off_yr + up(8 * n);
    const size_t off_ys = off_part + up(3 * kRankBlocks * sizeof(double)), off_out = off_ys + al;
    const size_t off_tmp = off_out + up((size_t)n_combos * sizeof(double));
    cudaError_t e = ensure(b.rank, off_tmp + tb);
    if (e != cudaSuccess) return status_from(e);
    char* base = (char*)b.rank.ptr;
    RankScratch s;
    s.keys[0] = base + off_k0;
    s.keys[1] = base + off_k1;
    s.ids[0] = (int32_t*)(base + off_i0);
    s.ids[1] = (int32_t*)(base + off_i1);
    s.start = (int32_t*)(base + off_st);
    s.end_of = (int32_t*)(base + off_en);
    s.ycr = (double*)(base + off_ycr);
    double* yrank = (double*)(base + off_yr);
    s.partial = (double*)(base + off_part);
    s.ystat = (double*)(base + off_ys);
    double* d_out = (double*)(base + off_out);
    s.temp = base + off_tmp;
    s.temp_bytes = tb;

    ColumnStats cs;
    const bool centred = center != 0;
    std::vector<double> means;
    bool any_pair = false;
    for (int64_t c = 0; c < n_combos; ++c) any_pair |= feat_b[c] >= 0;
    if (centred && any_pair) {
        int stc = compute_column_stats(b, false, cs);  // means of the raw columns at [c*4 + 3]
        if (stc != GAFIME_SUCCESS) return stc;
        means.resize((size_t)b.f);
        std::vector<double> col((size_t)b.f * 4);
        e = cudaMemcpyAsync(col.data(), cs.d_col, col.size() * sizeof(double), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return status_from(e);
        for (int64_t c = 0; c < b.f; ++c) means[(size_t)c] = col[(size_t)c * 4 + 3];
    }
    const unsigned g = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * b.sm_count));

    // target ranks
    const float* y = b.d_data + b.f * b.ld;
    fill_keys_kernel<uint32_t><<<g, 256, 0, st>>>(y, 0, n, 0, -1, 0, op, div_eps, 0.0, 0.0,
                                                  (uint32_t*)s.keys[0], s.ids[0]);
    e = sort_and_runs<uint32_t>(s, n, b.sm_count, st);
    if (e != cudaSuccess) return status_from(e);
    rank_sums_kernel<<<kRankBlocks, kRankThreads, 0, st>>>(s.start, s.end_of, s.ids[1], n, nullptr, yrank, s.partial);
    rank_final_kernel<<<1, 1, 0, st>>>(s.partial, kRankBlocks, n, 0, s.ystat, nullptr);
    centre_kernel<<<g, 256, 0, st>>>(yrank, n, s.ystat, s.ycr);
    e = cudaGetLastError();
    if (e != cudaSuccess) return status_from(e);

    for (int64_t c = 0; c < n_combos; ++c) {
        const int a = feat_a[c], bb = feat_b[c];
        const bool wide = bb >= 0 && centred;  // fp64 centred product: 64-bit keys
        if (wide) {
            fill_keys_kernel<uint64_t><<<g, 256, 0, st>>>(b.d_data, b.ld, n, a, bb, 2, op, div_eps,
                                                          means[(size_t)a], means[(size_t)bb],
                                                          (uint64_t*)s.keys[0], s.ids[0]);
            e = sort_and_runs<uint64_t>(s, n, b.sm_count, st);
        } else {
            fill_keys_kernel<uint32_t><<<g, 256, 0, st>>>(b.d_data, b.ld, n, a, bb, bb < 0 ? 0 : 1, op, div_eps,
                                                          0.0, 0.0, (uint32_t*)s.keys[0], s.ids[0]);
            e = sort_and_runs<uint32_t>(s, n, b.sm_count, st);
        }
        if (e != cudaSuccess) return status_from(e);
        rank_sums_kernel<<<kRankBlocks, kRankThreads, 0, st>>>(s.start, s.end_of, s.ids[1], n, s.ycr, nullptr,
                                                               s.partial);
        rank_final_kernel<<<1, 1, 0, st>>>(s.partial, kRankBlocks, n, 1, s.ystat, d_out + c);
    }
    e = cudaGetLastError();
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(out, d_out, (size_t)n_combos * sizeof(double), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return status_from(e);
}

}  // namespace gafime

using namespace gafime;

extern "C" int gafime_spearman_scores(ContiguousBucket bucket, const int32_t* feat_a, const int32_t* feat_b,
                                      int64_t n_combos, int interact_type, int center, float div_eps,
                                      double* out_scores) {
    if (!bucket || n_combos < 0 || (n_combos > 0 && (!feat_a || !feat_b || !out_scores)))
        return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    if (interact_type < GAFIME_INTERACT_MULT || interact_type > GAFIME_INTERACT_DIV) return GAFIME_ERROR_INVALID_ARGS;
    if (b->n > 0x7fffffff) return GAFIME_ERROR_INVALID_ARGS;
    for (int64_t c = 0; c < n_combos; ++c)
        if (feat_a[c] < 0 || feat_a[c] >= b->f || feat_b[c] >= b->f) return GAFIME_ERROR_INVALID_ARGS;
    if (n_combos == 0) return GAFIME_SUCCESS;
    cudaSetDevice(b->device);
    bool finite = true;
    int st = check_finite(*b, &finite);
    if (st != GAFIME_SUCCESS) return st;
    if (!finite) return GAFIME_ERROR_INVALID_ARGS;
    return spearman_scores(*b, feat_a, feat_b, n_combos, interact_type, center, div_eps, out_scores);
}
