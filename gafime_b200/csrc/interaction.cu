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
#include <stdint.h>

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
