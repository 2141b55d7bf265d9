// moments.cu -- CUDA-core pair-moment kernel for every operator.
//
// For a tile of 64 x 64 column pairs (i in the A block, j in the B block) and a
// span of rows, each CTA accumulates three moments of x = a * g(b):
//     S1 = sum x,   S2 = sum x^2,   S3 = sum x * ycen      (ycen = y - mean y)
// with g = identity (multiply; add and subtract reuse S1 = sum a*b) or
// g(b) = 1 / safe(b) (divide, safe(b) = |b| < eps ? copysign(eps, b) : b,
// cpu_backend.cpp:93-94).  For multiply x = fl32(a*b) exactly as the reference
// forms it (cpu_backend.cpp:100-101); for divide x = a * fl32(1/safe(b)).
//
// Data path: column-major fp32 X in HBM -> cp.async (16 B, coalesced, 4 stages)
// -> shared memory [col][32 rows + 4 pad] -> each thread owns a 4 x 4 pair
// micro-tile (A cols ty+16m, B cols tx+16q) and reads float4 runs of 4 rows.
// Sums run in fp32 for 256 rows, then are flushed into fp64 registers; the fp64
// partials of each (tile, row split) are written to HBM and combined in a fixed
// order by the scoring epilogue (deterministic, no atomics).
#include <cuda_runtime.h>
#include <stdint.h>

#include "engine.h"

namespace gafime {

namespace {

constexpr int kThreads = 256;
constexpr int kRows = 32;           // rows per pipeline stage
constexpr int kColStride = 36;      // floats per column in smem (bank-conflict-free float4 reads)
constexpr int kStages = 4;
constexpr int kFlushChunks = 8;     // fp32 span = 256 rows

struct __align__(16) Stage {
    float a[kTile * kColStride];
    float b[kTile * kColStride];
    float y[kRows];
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Issue the copies of one 32-row chunk: 64 A columns, 64 B columns, 32 ycen.
// Columns at or beyond f are zero-filled (their pairs are masked later).
__device__ __forceinline__ void load_stage(Stage& st, const float* __restrict__ x, int64_t ld,
                                           const float* __restrict__ ycen, int64_t f, int a0,
                                           int b0, int64_t r0, int tid) {
    #pragma unroll
    for (int h = 0; h < 4; ++h) {
        int g = tid + h * kThreads;          // 0..1023: 512 A granules then 512 B granules
        int side = g >> 9;
        int gg = g & 511;
        int col = gg >> 3, part = gg & 7;
        int gc = (side ? b0 : a0) + col;
        bool ok = gc < f;
        const float* src = x + (int64_t)(ok ? gc : 0) * ld + r0 + 4 * part;
        float* dst = (side ? st.b : st.a) + col * kColStride + 4 * part;
        cp_async16(dst, src, ok ? 16 : 0);
    }
    if (tid < kRows / 4) cp_async16(st.y + 4 * tid, ycen + r0 + 4 * tid, 16);
}

template <bool kRecip>
__global__ void __launch_bounds__(kThreads, 1) pair_moments_kernel(
    const float* __restrict__ x, int64_t ld, const float* __restrict__ ycen, int64_t f,
    const TileCoord* __restrict__ tiles, int n_tiles, int64_t rows_per_split, float eps,
    double* __restrict__ moments) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Stage* stages = reinterpret_cast<Stage*>(smem_raw);

    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int t = blockIdx.x, split = blockIdx.y;
    const TileCoord tc = tiles[t];
    const int a0 = tc.bi * kTile, b0 = tc.bj * kTile;
    const int64_t r_begin = (int64_t)split * rows_per_split;
    int64_t r_end = r_begin + rows_per_split;
    if (r_end > ld) r_end = ld;
    const int n_chunks = r_end > r_begin ? (int)((r_end - r_begin) / kRows) : 0;

    float s1[4][4], s2[4][4], s3[4][4];
    double d1[4][4], d2[4][4], d3[4][4];
    #pragma unroll
    for (int m = 0; m < 4; ++m)
        #pragma unroll
        for (int q = 0; q < 4; ++q) {
            s1[m][q] = s2[m][q] = s3[m][q] = 0.0f;
            d1[m][q] = d2[m][q] = d3[m][q] = 0.0;
        }

    // prologue: stages 0 .. kStages-2
    #pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < n_chunks) load_stage(stages[s], x, ld, ycen, f, a0, b0, r_begin + (int64_t)s * kRows, tid);
        cp_async_commit();
    }

    for (int c = 0; c < n_chunks; ++c) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        {
            int nc = c + kStages - 1;
            if (nc < n_chunks)
                load_stage(stages[nc % kStages], x, ld, ycen, f, a0, b0, r_begin + (int64_t)nc * kRows, tid);
            cp_async_commit();
        }
        Stage& st = stages[c % kStages];
        if (kRecip) {
            // g(b) = 1 / safe(b), computed once per element for the whole CTA.
            #pragma unroll
            for (int h = 0; h < (kTile * kRows) / kThreads; ++h) {
                int e = tid + h * kThreads;
                int col = e >> 5, r = e & 31;
                float v = st.b[col * kColStride + r];
                float d = fabsf(v) < eps ? copysignf(eps, v) : v;
                st.b[col * kColStride + r] = __frcp_rn(d);
            }
            __syncthreads();
        }
        #pragma unroll 2
        for (int r4 = 0; r4 < kRows / 4; ++r4) {
            const float4 yv = *reinterpret_cast<const float4*>(st.y + 4 * r4);
            float4 av[4];
            #pragma unroll
            for (int m = 0; m < 4; ++m)
                av[m] = *reinterpret_cast<const float4*>(st.a + (ty + 16 * m) * kColStride + 4 * r4);
            #pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 bv = *reinterpret_cast<const float4*>(st.b + (tx + 16 * q) * kColStride + 4 * r4);
                #pragma unroll
                for (int m = 0; m < 4; ++m) {
                    float v;
                    v = __fmul_rn(av[m].x, bv.x);
                    s1[m][q] += v; s2[m][q] = fmaf(v, v, s2[m][q]); s3[m][q] = fmaf(v, yv.x, s3[m][q]);
                    v = __fmul_rn(av[m].y, bv.y);
                    s1[m][q] += v; s2[m][q] = fmaf(v, v, s2[m][q]); s3[m][q] = fmaf(v, yv.y, s3[m][q]);
                    v = __fmul_rn(av[m].z, bv.z);
                    s1[m][q] += v; s2[m][q] = fmaf(v, v, s2[m][q]); s3[m][q] = fmaf(v, yv.z, s3[m][q]);
                    v = __fmul_rn(av[m].w, bv.w);
                    s1[m][q] += v; s2[m][q] = fmaf(v, v, s2[m][q]); s3[m][q] = fmaf(v, yv.w, s3[m][q]);
                }
            }
        }
        if ((c + 1) % kFlushChunks == 0 || c + 1 == n_chunks) {
            #pragma unroll
            for (int m = 0; m < 4; ++m)
                #pragma unroll
                for (int q = 0; q < 4; ++q) {
                    d1[m][q] += (double)s1[m][q];
                    d2[m][q] += (double)s2[m][q];
                    d3[m][q] += (double)s3[m][q];
                    s1[m][q] = s2[m][q] = s3[m][q] = 0.0f;
                }
        }
    }
    cp_async_wait<0>();

    double* out = moments + ((int64_t)split * n_tiles + t) * 3 * kTilePairs;
    #pragma unroll
    for (int m = 0; m < 4; ++m)
        #pragma unroll
        for (int q = 0; q < 4; ++q) {
            int li = ty + 16 * m, lj = tx + 16 * q;
            int e = li * kTile + lj;
            out[e] = d1[m][q];
            out[kTilePairs + e] = d2[m][q];
            out[2 * kTilePairs + e] = d3[m][q];
        }
}

}  // namespace

cudaError_t launch_pair_moments(const float* d_x, int64_t ld, const float* d_ycen, int64_t f,
                                const TileCoord* d_tiles, int n_tiles, int splits,
                                int64_t rows_per_split, bool recip, float eps, double* d_moments,
                                cudaStream_t stream) {
    if (n_tiles <= 0) return cudaSuccess;
    if (rows_per_split % kRows != 0) return cudaErrorInvalidValue;
    const size_t smem = sizeof(Stage) * kStages;
    dim3 grid((unsigned)n_tiles, (unsigned)splits);
    if (recip) {
        cudaFuncSetAttribute(pair_moments_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        pair_moments_kernel<true><<<grid, kThreads, smem, stream>>>(d_x, ld, d_ycen, f, d_tiles, n_tiles,
                                                                    rows_per_split, eps, d_moments);
    } else {
        cudaFuncSetAttribute(pair_moments_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        pair_moments_kernel<false><<<grid, kThreads, smem, stream>>>(d_x, ld, d_ycen, f, d_tiles, n_tiles,
                                                                     rows_per_split, eps, d_moments);
    }
    return cudaGetLastError();
}

}  // namespace gafime
