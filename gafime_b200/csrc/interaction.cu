// interaction.cu -- the legacy interaction materialiser of the reference ABI.
//
// gafime_feature_interaction_cuda (interfaces.h:392-401; semantics of the reference kernel,
// src/cuda/kernels.cu:1646-1676):
//   out[i, c] = X[i, f]                                   for a one-feature combo c = {f}
//   out[i, c] = prod over f in c of fl32(X[i, f] - means[f])   otherwise, in combo order
// X and out are row-major (row i at X + i * F, out + i * n_combos); feature ids outside
// [0, F) are skipped, so an empty combo yields 1.  The reference's NativeCudaBackend binds
// this symbol when it loads the library (native_cuda_backend.py:113-124) and calls it to
// build single interaction vectors (native_cuda_backend.py:230-258) and for its legacy
// mutual-information route (native_cuda_backend.py:420-468).  Synchronous, host buffers in
// and out, like the reference.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>

#include "engine.h"

namespace gafime {
namespace {

// one thread per (row, combo); threads of a warp take consecutive combos of one row, so
// the output row is written coalesced and the row of X is read through L1
__global__ void __launch_bounds__(256) interaction_kernel(const float* __restrict__ X, const float* __restrict__ means,
                                                          float* __restrict__ out, const int32_t* __restrict__ idx,
                                                          const int32_t* __restrict__ off, int32_t n, int32_t f,
                                                          int32_t n_combos) {
    const int32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t i = (int64_t)blockIdx.y * blockDim.y + threadIdx.y;
    if (c >= n_combos || i >= n) return;
    const int32_t start = off[c], end = off[c + 1], size = end - start;
    const float* row = X + i * f;
    float prod = 1.0f;
    for (int32_t j = start; j < end; ++j) {
        const int32_t feat = idx[j];
        if (feat < 0 || feat >= f) continue;
        const float v = row[feat];
        if (size == 1) prod = v;
        else prod = __fmul_rn(prod, __fsub_rn(v, means[feat]));
    }
    out[i * n_combos + c] = prod;
}

}  // namespace
}  // namespace gafime

using namespace gafime;

extern "C" int gafime_feature_interaction_cuda(const float* X, const float* means, float* output,
                                               const int32_t* combo_indices, const int32_t* combo_offsets,
                                               int32_t n_samples, int32_t n_features, int32_t n_combos) {
    if (!X || !means || !output || !combo_indices || !combo_offsets) return GAFIME_ERROR_INVALID_ARGS;
    if (n_samples <= 0 || n_features <= 0 || n_combos <= 0) return GAFIME_ERROR_INVALID_ARGS;
    // the offsets must describe ranges of combo_indices: start at >= 0 and never decrease
    if (combo_offsets[0] < 0) return GAFIME_ERROR_INVALID_ARGS;
    for (int32_t c = 0; c < n_combos; ++c)
        if (combo_offsets[c + 1] < combo_offsets[c]) return GAFIME_ERROR_INVALID_ARGS;
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;

    const size_t x_bytes = (size_t)n_samples * n_features * sizeof(float);
    const size_t out_bytes = (size_t)n_samples * n_combos * sizeof(float);
    const size_t n_idx = (size_t)combo_offsets[n_combos] > 0 ? (size_t)combo_offsets[n_combos] : 1;
    float *d_x = nullptr, *d_means = nullptr, *d_out = nullptr;
    int32_t *d_idx = nullptr, *d_off = nullptr;
    cudaError_t e = cudaMalloc(&d_x, x_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&d_means, (size_t)n_features * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&d_out, out_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&d_idx, n_idx * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMalloc(&d_off, ((size_t)n_combos + 1) * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemcpy(d_x, X, x_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d_means, means, (size_t)n_features * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && combo_offsets[n_combos] > 0)
        e = cudaMemcpy(d_idx, combo_indices, (size_t)combo_offsets[n_combos] * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(d_off, combo_offsets, ((size_t)n_combos + 1) * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        const dim3 block(32, 8);
        const dim3 grid((unsigned)((n_combos + 31) / 32), (unsigned)((n_samples + 7) / 8));
        interaction_kernel<<<grid, block>>>(d_x, d_means, d_out, d_idx, d_off, n_samples, n_features, n_combos);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(output, d_out, out_bytes, cudaMemcpyDeviceToHost);
    const bool oom = e == cudaErrorMemoryAllocation;
    cudaFree(d_x);
    cudaFree(d_means);
    cudaFree(d_out);
    cudaFree(d_idx);
    cudaFree(d_off);
    if (e == cudaSuccess) return GAFIME_SUCCESS;
    return oom ? GAFIME_ERROR_OUT_OF_MEMORY : GAFIME_ERROR_KERNEL_FAILED;
}

// ---- gafime_pearson_cuda ----------------------------------------------------------
//
// Declared by the reference (interfaces.h:420-425) without a GPU implementation; the
// arithmetic follows its CPU twin gafime_pearson_cpu (cpu_backend.cpp:374-411): fp64
// sums, r = (Sxy - Sx*my) / sqrt((Sxx - Sx*mx)(Syy - Sy*my)), 0 when a variance is <= 0,
// cast to float.  Sums here are reduced in a fixed order (deterministic).

namespace gafime {
namespace {

constexpr int kPearsonBlocks = 256;

__global__ void __launch_bounds__(256) pearson_sums_kernel(const float* __restrict__ x, const float* __restrict__ y,
                                                           int32_t n, double* __restrict__ part /*[blocks][5]*/) {
    __shared__ double red[8][5];
    double s[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
        const double xi = x[i], yi = y[i];
        s[0] += xi;
        s[1] += yi;
        s[2] += xi * xi;
        s[3] += yi * yi;
        s[4] += xi * yi;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    #pragma unroll
    for (int m = 0; m < 5; ++m)
        for (int o = 16; o > 0; o >>= 1) s[m] += __shfl_down_sync(0xffffffffu, s[m], o);
    if (lane == 0)
        #pragma unroll
        for (int m = 0; m < 5; ++m) red[warp][m] = s[m];
    __syncthreads();
    if (threadIdx.x < 5) {
        double t = red[0][threadIdx.x];
        for (int w = 1; w < 8; ++w) t += red[w][threadIdx.x];
        part[blockIdx.x * 5 + threadIdx.x] = t;
    }
}

__global__ void pearson_finish_kernel(const double* __restrict__ part, int blocks, int32_t n, float* out) {
    double s[5] = {0.0, 0.0, 0.0, 0.0, 0.0};
    for (int b = 0; b < blocks; ++b)
        for (int m = 0; m < 5; ++m) s[m] += part[b * 5 + m];
    const double mx = s[0] / n, my = s[1] / n;
    const double vx = s[2] - s[0] * mx, vy = s[3] - s[1] * my, cov = s[4] - s[0] * my;
    *out = (vx <= 0.0 || vy <= 0.0) ? 0.0f : (float)(cov / sqrt(vx * vy));
}

}  // namespace
}  // namespace gafime

extern "C" int gafime_pearson_cuda(const float* x, const float* y, int32_t n, float* result_out) {
    if (!x || !y || !result_out || n <= 0) return GAFIME_ERROR_INVALID_ARGS;
    int dev_count = 0;
    if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;
    const int blocks = (int)std::min<int64_t>(kPearsonBlocks, ((int64_t)n + 255) / 256);
    float *d_x = nullptr, *d_y = nullptr, *d_r = nullptr;
    double* d_part = nullptr;
    cudaError_t e = cudaMalloc(&d_x, (size_t)n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&d_y, (size_t)n * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&d_part, (size_t)blocks * 5 * sizeof(double));
    if (e == cudaSuccess) e = cudaMalloc(&d_r, sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(d_x, x, (size_t)n * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(d_y, y, (size_t)n * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        pearson_sums_kernel<<<blocks, 256>>>(d_x, d_y, n, d_part);
        pearson_finish_kernel<<<1, 1>>>(d_part, blocks, n, d_r);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(result_out, d_r, sizeof(float), cudaMemcpyDeviceToHost);
    const bool oom = e == cudaErrorMemoryAllocation;
    cudaFree(d_x);
    cudaFree(d_y);
    cudaFree(d_part);
    cudaFree(d_r);
    if (e == cudaSuccess) return GAFIME_SUCCESS;
    return oom ? GAFIME_ERROR_OUT_OF_MEMORY : GAFIME_ERROR_KERNEL_FAILED;
}
