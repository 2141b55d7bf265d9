// bucket.cu -- device queries, the contiguous bucket (reference ABI), the legacy
// single-pair 12-stat kernel, and the fp64 column statistics every all-pairs
// scoring pass starts from.
//
// Reference behaviour mirrored here:
//   gafime_contiguous_bucket_alloc/upload/compute/free/info  kernels.cu:2183-2556
//   apply_op / combine (accurate libm forms of cpu_backend.cpp:30-103)
//   12-stat layout, NaN-row skip, fold split              interfaces.h:110-123,
//                                                         cpu_backend.cpp:261-293
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <new>
#include <vector>

#include "engine.h"

namespace gafime {

int status_from(cudaError_t e) {
    if (e == cudaSuccess) return GAFIME_SUCCESS;
    if (e == cudaErrorMemoryAllocation) return GAFIME_ERROR_OUT_OF_MEMORY;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;
    return GAFIME_ERROR_KERNEL_FAILED;
}

cudaError_t ensure(DeviceBuf& b, size_t bytes) {
    if (b.bytes >= bytes && b.ptr) return cudaSuccess;
    if (b.ptr) {
        // Growing: queued kernels may still read the old buffer, so drain the device
        // before freeing it.  Happens only when a call needs more scratch than any before.
        cudaDeviceSynchronize();
        cudaFree(b.ptr);
        b.ptr = nullptr;
        b.bytes = 0;
    }
    size_t want = bytes < 256 ? 256 : bytes;
    cudaError_t e = cudaMalloc(&b.ptr, want);
    if (e == cudaSuccess) b.bytes = want;
    return e;
}

static void release(DeviceBuf& b) {
    if (b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.bytes = 0;
}

// ------------------------------------------------------------- unary / combine --

// Unary operators with the accurate math functions of the CPU reference
// (cpu_backend.cpp:30-77); the 12-stat parity target is that CPU library.
__device__ __forceinline__ float apply_op(float x, int op) {
    switch (op) {
        case GAFIME_OP_LOG: return logf(fabsf(x) + 1e-8f);
        case GAFIME_OP_EXP: return expf(fminf(fmaxf(x, -20.0f), 20.0f));
        case GAFIME_OP_SQRT: return sqrtf(fabsf(x));
        case GAFIME_OP_TANH: {
            float c = fminf(fmaxf(x, -10.0f), 10.0f);
            float e2 = expf(2.0f * c);
            return (e2 - 1.0f) / (e2 + 1.0f);
        }
        case GAFIME_OP_SIGMOID: {
            float c = fminf(fmaxf(x, -20.0f), 20.0f);
            return 1.0f / (1.0f + expf(-c));
        }
        case GAFIME_OP_SQUARE: return x * x;
        case GAFIME_OP_NEGATE: return -x;
        case GAFIME_OP_ABS: return fabsf(x);
        case GAFIME_OP_INVERSE: return 1.0f / (fabsf(x) < 1e-8f ? copysignf(1e-8f, x) : x);
        case GAFIME_OP_CUBE: return x * x * x;
        case GAFIME_OP_ROLLING_MEAN:
        case GAFIME_OP_ROLLING_STD: return __int_as_float(0x7fc00000);  // NaN: row skipped
        case GAFIME_OP_IDENTITY:
        default: return x;
    }
}

__device__ __forceinline__ float combine_op(float a, float b, int t) {
    switch (t) {
        case GAFIME_INTERACT_ADD: return a + b;
        case GAFIME_INTERACT_SUB: return a - b;
        case GAFIME_INTERACT_DIV: return a / (fabsf(b) < 1e-8f ? copysignf(1e-8f, b) : b);
        case GAFIME_INTERACT_MAX: return fmaxf(a, b);
        case GAFIME_INTERACT_MIN: return fminf(a, b);
        case GAFIME_INTERACT_MULT:
        default: return __fmul_rn(a, b);
    }
}

// --------------------------------------------------------------- reductions --

// Fixed-order block reduction of NV doubles per thread (blockDim.x == 256).
template <int NV>
__device__ __forceinline__ void block_reduce_fixed(double (&v)[NV], double* smem /*[NV*256]*/) {
    const int t = threadIdx.x;
    #pragma unroll
    for (int m = 0; m < NV; ++m) smem[m * 256 + t] = v[m];
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (t < s) {
            #pragma unroll
            for (int m = 0; m < NV; ++m) smem[m * 256 + t] += smem[m * 256 + t + s];
        }
        __syncthreads();
    }
    #pragma unroll
    for (int m = 0; m < NV; ++m) v[m] = smem[m * 256];
}

// --------------------------------------------------- legacy single-pair stats --

constexpr int kLegacyBlocks = 296;

__global__ void __launch_bounds__(256) legacy_pair_stats_kernel(
    const float* __restrict__ data, const uint8_t* __restrict__ mask, int64_t n, int64_t ld,
    int64_t f, int fa, int fb, int op_a, int op_b, int interact, int val_fold_id,
    double* __restrict__ partial /*[gridDim.x][12]*/) {
    __shared__ double red[12 * 256];
    const float* ca = data + (int64_t)fa * ld;
    const float* cb = data + (int64_t)fb * ld;
    const float* y = data + f * ld;
    double acc[12];
    #pragma unroll
    for (int m = 0; m < 12; ++m) acc[m] = 0.0;
    for (int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x; r < n; r += (int64_t)gridDim.x * 256) {
        float x = combine_op(apply_op(ca[r], op_a), apply_op(cb[r], op_b), interact);
        float yv = y[r];
        if (isnan(x) || isnan(yv)) continue;
        double xd = x, yd = yv;
        int o = (mask[r] == val_fold_id) ? 6 : 0;
        #pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (o == 6 * h) {
                acc[6 * h + 0] += 1.0;
                acc[6 * h + 1] += xd;
                acc[6 * h + 2] += yd;
                acc[6 * h + 3] += xd * xd;
                acc[6 * h + 4] += yd * yd;
                acc[6 * h + 5] += xd * yd;
            }
        }
    }
    block_reduce_fixed<12>(acc, red);
    if (threadIdx.x == 0) {
        #pragma unroll
        for (int m = 0; m < 12; ++m) partial[blockIdx.x * 12 + m] = acc[m];
    }
}

__global__ void sum_partials_kernel(const double* __restrict__ partial, int n_part, int width,
                                    double* __restrict__ out) {
    int m = threadIdx.x;
    if (m >= width) return;
    double s = 0.0;
    for (int p = 0; p < n_part; ++p) s += partial[p * width + m];
    out[m] = s;
}

// ------------------------------------------------------------ column stats --

// Partial sums over one row split of one column: [0] sum x, [1] sum x^2,
// [2] sum x*ycen (when ycen != nullptr).
__global__ void __launch_bounds__(256) col_partial_kernel(
    const float* __restrict__ x, int64_t ld, int64_t n, const float* __restrict__ ycen,
    int64_t span, double* __restrict__ part /*[cols][splits][3]*/) {
    __shared__ double red[3 * 256];
    const int c = blockIdx.x, s = blockIdx.y, splits = gridDim.y;
    const float* col = x + (int64_t)c * ld;
    int64_t r0 = (int64_t)s * span;
    int64_t r1 = r0 + span < n ? r0 + span : n;
    double v[3] = {0.0, 0.0, 0.0};
    // rows r0 + tid, + 256, ... in order; each run of 8 issues its loads before any use
    constexpr int kRun = 8;
    for (int64_t base = r0 + threadIdx.x; base < r1; base += 256 * kRun) {
        float xv[kRun], yv[kRun];
        #pragma unroll
        for (int i = 0; i < kRun; ++i) {
            const int64_t r = base + 256 * i;
            xv[i] = r < r1 ? __ldg(col + r) : 0.f;
            yv[i] = (ycen && r < r1) ? __ldg(ycen + r) : 0.f;
        }
        #pragma unroll
        for (int i = 0; i < kRun; ++i) {
            if (base + 256 * i < r1) {
                const double a = xv[i];
                v[0] += a;
                v[1] += a * a;
                if (ycen) v[2] += a * (double)yv[i];
            }
        }
    }
    block_reduce_fixed<3>(v, red);
    if (threadIdx.x == 0) {
        double* o = part + ((int64_t)c * splits + s) * 3;
        o[0] = v[0];
        o[1] = v[1];
        o[2] = v[2];
    }
}

// colstats[c*4 + {0,1,2,3}] = {sum, sumsq, sum x*ycen, mean}
__global__ void col_combine_kernel(const double* __restrict__ part, int cols, int splits,
                                   int64_t n, double* __restrict__ colstats) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    double v[3] = {0.0, 0.0, 0.0};
    for (int s = 0; s < splits; ++s)
        for (int m = 0; m < 3; ++m) v[m] += part[((int64_t)c * splits + s) * 3 + m];
    colstats[c * 4 + 0] = v[0];
    colstats[c * 4 + 1] = v[1];
    colstats[c * 4 + 2] = v[2];
    colstats[c * 4 + 3] = v[0] / (double)n;
}

// col_combine_kernel with one block per column: thread t adds splits t, t + 256, ... in
// order, then a fixed-order tree over the threads (deterministic); many splits (a single
// tall column) no longer run through one thread.
__global__ void __launch_bounds__(256) col_combine_block_kernel(const double* __restrict__ part, int splits,
                                                                int64_t n, double* __restrict__ colstats) {
    __shared__ double red[3 * 256];
    const int c = blockIdx.x;
    double v[3] = {0.0, 0.0, 0.0};
    for (int s = threadIdx.x; s < splits; s += 256)
        for (int m = 0; m < 3; ++m) v[m] += part[((int64_t)c * splits + s) * 3 + m];
    block_reduce_fixed<3>(v, red);
    if (threadIdx.x != 0) return;
    colstats[c * 4 + 0] = v[0];
    colstats[c * 4 + 1] = v[1];
    colstats[c * 4 + 2] = v[2];
    colstats[c * 4 + 3] = v[0] / (double)n;
}

// ystats = {n, sum y, var_y, mean y} from the target column's (sum, sumsq).
// var_y = syy - sy^2/n as native_cuda_backend.py:481 and gafime_core.cpp:496.
__global__ void ystats_kernel(const double* __restrict__ ycol, int64_t n, double* __restrict__ ystats) {
    double dn = (double)n, sy = ycol[0], syy = ycol[1];
    double mean = sy / dn;
    ystats[0] = dn;
    ystats[1] = sy;
    ystats[2] = syy - sy * mean;
    ystats[3] = mean;
}

__global__ void ycen_kernel(const float* __restrict__ y, int64_t n, int64_t ld,
                            const double* __restrict__ ystats, float* __restrict__ ycen) {
    double mean = ystats[3];
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < ld;
         r += (int64_t)gridDim.x * blockDim.x)
        ycen[r] = r < n ? (float)((double)y[r] - mean) : 0.0f;
}

// Centred copy fl32(x - mean) in the padded layout (pad rows stay zero).
__global__ void xcen_kernel(const float* __restrict__ x, int64_t ld, int64_t n, int64_t f,
                            const double* __restrict__ colstats, float* __restrict__ xc) {
    int64_t total = f * ld;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        int64_t c = e / ld, r = e - c * ld;
        xc[e] = r < n ? (float)((double)x[e] - colstats[c * 4 + 3]) : 0.0f;
    }
}

__global__ void finite_kernel(const float* __restrict__ x, int64_t cols, int64_t ld, int64_t n,
                              int* __restrict__ flag) {
    int64_t total = cols * ld;
    int bad = 0;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = e % ld;
        if (r < n && !isfinite(x[e])) bad = 1;
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

static int split_count(int64_t cols, int64_t n, int sm) {
    int64_t want = (16 * (int64_t)sm + cols - 1) / cols;  // ~16 CTAs per SM of column passes
    int64_t max_by_rows = (n + 4095) / 4096;
    if (want > max_by_rows) want = max_by_rows;
    if (want < 1) want = 1;
    if (want > 1024) want = 1024;
    return (int)want;
}

// Column partial sums + combine for `cols` columns of `x` into colstats[cols*4].
static cudaError_t column_sums(Bucket& b, const float* x, int64_t cols, const float* ycen,
                               double* colstats) {
    int splits = split_count(cols, b.n, b.sm_count);
    int64_t span = (b.n + splits - 1) / splits;
    span = (span + 255) / 256 * 256;
    cudaError_t e = ensure(b.stats_part, (size_t)cols * splits * 3 * sizeof(double));
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)cols, (unsigned)splits);
    col_partial_kernel<<<grid, 256, 0, b.stream>>>(x, b.ld, b.n, ycen, span,
                                                   (double*)b.stats_part.ptr);
    col_combine_block_kernel<<<(unsigned)cols, 256, 0, b.stream>>>((const double*)b.stats_part.ptr, splits, b.n,
                                                                    colstats);
    return cudaGetLastError();
}

int compute_column_stats(Bucket& b, bool centred, ColumnStats& out, bool x_sums) {
    // stats buffer: [f*4] column stats, [4] y column sums, [4] ystats
    cudaError_t e = ensure(b.stats, (size_t)(b.f * 4 + 8) * sizeof(double));
    if (e == cudaSuccess) {
        size_t need = (size_t)std::max<int64_t>(1 * split_count(1, b.n, b.sm_count),
                                                b.f * split_count(b.f, b.n, b.sm_count));
        e = ensure(b.stats_part, need * 3 * sizeof(double));
    }
    if (e == cudaSuccess) e = ensure(b.ycen, (size_t)b.ld * sizeof(float));
    if (e != cudaSuccess) return status_from(e);
    double* colstats = (double*)b.stats.ptr;
    double* ycol = colstats + b.f * 4;
    double* ystats = ycol + 4;
    const float* y = b.d_data + b.f * b.ld;
    float* ycen = (float*)b.ycen.ptr;
    int blocks = 4 * b.sm_count;

    e = column_sums(b, y, 1, nullptr, ycol);
    if (e != cudaSuccess) return status_from(e);
    ystats_kernel<<<1, 1, 0, b.stream>>>(ycol, b.n, ystats);
    ycen_kernel<<<blocks, 256, 0, b.stream>>>(y, b.n, b.ld, ystats, ycen);
    const float* xs = b.d_data;
    if (centred) {
        e = ensure(b.xcen, (size_t)b.f * b.ld * sizeof(float));
        if (e != cudaSuccess) return status_from(e);
        e = column_sums(b, b.d_data, b.f, nullptr, colstats);  // means of raw columns
        if (e != cudaSuccess) return status_from(e);
        xcen_kernel<<<blocks, 256, 0, b.stream>>>(b.d_data, b.ld, b.n, b.f, colstats,
                                                   (float*)b.xcen.ptr);
        xs = (const float*)b.xcen.ptr;
    }
    if (x_sums) {
        e = column_sums(b, xs, b.f, ycen, colstats);
        if (e != cudaSuccess) return status_from(e);
    }
    out.d_col = colstats;
    out.d_y = ystats;
    out.d_x = xs;
    out.d_ycen = ycen;
    return GAFIME_SUCCESS;
}

// Whole-buffer check with float4 loads: pad rows are zero, so every element can be tested.
__global__ void finite4_kernel(const float4* __restrict__ x, int64_t n4, int* __restrict__ flag) {
    int bad = 0;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n4; e += (int64_t)gridDim.x * blockDim.x) {
        float4 v = x[e];
        bad |= !isfinite(v.x) | !isfinite(v.y) | !isfinite(v.z) | !isfinite(v.w);
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

cudaError_t launch_finite_check(const float* x, int64_t n_floats, int* flag, int blocks, cudaStream_t stream) {
    finite4_kernel<<<blocks, 256, 0, stream>>>((const float4*)x, n_floats / 4, flag);
    return cudaGetLastError();
}

// Checks the bucket's features and target once per upload (the result is kept until the
// next upload replaces the data).
int check_finite(Bucket& b, bool* all_finite) {
    if (b.finite_state >= 0) {
        *all_finite = b.finite_state == 1;
        return GAFIME_SUCCESS;
    }
    cudaError_t e = ensure(b.flags, 64);
    if (e != cudaSuccess) return status_from(e);
    int* flag = (int*)b.flags.ptr;
    cudaMemsetAsync(flag, 0, sizeof(int), b.stream);
    finite4_kernel<<<4 * b.sm_count, 256, 0, b.stream>>>((const float4*)b.d_data, (b.f + 1) * b.ld / 4, flag);
    int h = 0;
    e = cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, b.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return status_from(e);
    *all_finite = (h == 0);
    b.finite_state = *all_finite ? 1 : 0;
    return GAFIME_SUCCESS;
}

// Rows [0, n) of dst's column c are src column scol[c] at rows rows[r] (identity when rows is
// null); pad rows of dst stay zero.  blockIdx.y strides over dst's columns (features, then
// the target), blockIdx.x over rows.
__global__ void gather_rows_kernel(const float* __restrict__ src, int64_t src_ld, const int32_t* __restrict__ scol,
                                   int64_t n_cols, const int64_t* __restrict__ rows, int64_t n,
                                   float* __restrict__ dst, int64_t dst_ld) {
    for (int64_t c = blockIdx.y; c < n_cols; c += gridDim.y) {
        const float* s = src + (int64_t)scol[c] * src_ld;
        float* d = dst + c * dst_ld;
        for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
            d[r] = s[rows ? rows[r] : r];
    }
}

__global__ void gather_mask_kernel(const uint8_t* __restrict__ src, const int64_t* __restrict__ rows, int64_t n,
                                   uint8_t* __restrict__ dst) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        dst[r] = src[rows ? rows[r] : r];
}

// Row-major rows [r0, r0 + rows) x F (row stride F) -> the bucket's column-major layout.
// 32 x 32 tiles through shared memory: coalesced reads along the row, coalesced writes
// along the column.
__global__ void __launch_bounds__(256) rows_to_columns_kernel(const float* __restrict__ src, int64_t rows,
                                                              int64_t f, float* __restrict__ dst, int64_t ld,
                                                              int64_t r0) {
    __shared__ float tile[32][33];
    const int64_t c_base = (int64_t)blockIdx.x * 32, r_base = (int64_t)blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (int k = ty; k < 32; k += 8) {
        const int64_t r = r_base + k, c = c_base + tx;
        tile[k][tx] = (r < rows && c < f) ? src[r * f + c] : 0.f;
    }
    __syncthreads();
    for (int k = ty; k < 32; k += 8) {
        const int64_t c = c_base + k, r = r_base + tx;
        if (c < f && r < rows) dst[c * ld + r0 + r] = tile[tx][k];
    }
}

}  // namespace gafime

using namespace gafime;

// ================================================================== C ABI ====

extern "C" {

int gafime_cuda_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n > 0 ? 1 : 0;
}

int gafime_select_device(int device_id) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;
    if (device_id < 0 || device_id >= n) return GAFIME_ERROR_INVALID_ARGS;
    return status_from(cudaSetDevice(device_id));
}

int gafime_get_device_info(int device_id, char* name_out, int* memory_mb_out,
                           int* compute_cap_major_out, int* compute_cap_minor_out) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;
    if (device_id < 0 || device_id >= n) return GAFIME_ERROR_INVALID_ARGS;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device_id) != cudaSuccess) return GAFIME_ERROR_KERNEL_FAILED;
    if (name_out) {
        strncpy(name_out, p.name, 255);
        name_out[255] = '\0';
    }
    if (memory_mb_out) *memory_mb_out = (int)(p.totalGlobalMem / (1024 * 1024));
    if (compute_cap_major_out) *compute_cap_major_out = p.major;
    if (compute_cap_minor_out) *compute_cap_minor_out = p.minor;
    return GAFIME_SUCCESS;
}

int gafime_get_gpu_config(int* block_size_out, int* max_blocks_out, int* sm_count_out,
                          int* compute_major_out, int* compute_minor_out, int* l2_cache_bytes_out,
                          char* gpu_name_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return GAFIME_ERROR_KERNEL_FAILED;
    if (block_size_out) *block_size_out = 256;
    if (max_blocks_out) *max_blocks_out = p.multiProcessorCount * 8;
    if (sm_count_out) *sm_count_out = p.multiProcessorCount;
    if (compute_major_out) *compute_major_out = p.major;
    if (compute_minor_out) *compute_minor_out = p.minor;
    if (l2_cache_bytes_out) *l2_cache_bytes_out = p.l2CacheSize;
    if (gpu_name_out) {
        strncpy(gpu_name_out, p.name, 255);
        gpu_name_out[255] = '\0';
    }
    return GAFIME_SUCCESS;
}

int gafime_tensor_core_available(int* precision_mode) {
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
        cudaGetLastError();
        if (precision_mode) *precision_mode = 0;
        return 0;
    }
    if (precision_mode) *precision_mode = major >= 10 ? 4 : 0;
    return major >= 10 ? 1 : 0;
}

int gafime_contiguous_bucket_alloc(int n_samples, int n_features, ContiguousBucket* bucket_out) {
    if (n_samples <= 0 || n_features <= 0 || !bucket_out) return GAFIME_ERROR_INVALID_ARGS;
    if (!gafime_cuda_available()) return GAFIME_ERROR_CUDA_NOT_AVAILABLE;
    Bucket* b = new (std::nothrow) Bucket();
    if (!b) return GAFIME_ERROR_OUT_OF_MEMORY;
    cudaGetDevice(&b->device);
    cudaDeviceGetAttribute(&b->sm_count, cudaDevAttrMultiProcessorCount, b->device);
    b->n = n_samples;
    b->f = n_features;
    b->ld = (b->n + kRowPad - 1) / kRowPad * kRowPad;
    size_t bytes = (size_t)(b->f + 1) * (size_t)b->ld * sizeof(float);
    cudaError_t e = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMallocHost(&b->h_pinned, 64 * sizeof(double));
    if (e == cudaSuccess) e = cudaMalloc(&b->d_data, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&b->d_mask, (size_t)b->n);
    if (e == cudaSuccess) e = cudaMemsetAsync(b->d_data, 0, bytes, b->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(b->d_mask, 0, (size_t)b->n, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) {
        int st = status_from(e);
        gafime_contiguous_bucket_free(b);
        cudaGetLastError();
        return st;
    }
    *bucket_out = b;
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_upload(ContiguousBucket bucket, const float* h_data,
                                    const uint8_t* h_mask) {
    if (!bucket || !h_data || !h_mask) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    cudaSetDevice(b->device);
    // One strided copy places every column (and y) at its padded offset.
    cudaError_t e = cudaMemcpy2DAsync(b->d_data, (size_t)b->ld * sizeof(float), h_data,
                                      (size_t)b->n * sizeof(float), (size_t)b->n * sizeof(float),
                                      (size_t)(b->f + 1), cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(b->d_mask, h_mask, (size_t)b->n, cudaMemcpyHostToDevice, b->stream);
    {
        // also after a failure: no copy from the caller's buffers is left in flight
        const cudaError_t es = cudaStreamSynchronize(b->stream);
        if (e == cudaSuccess) e = es;
    }
    if (e != cudaSuccess) return status_from(e);
    // validate the new data at ingest: the all-pairs calls accept finite input only
    b->finite_state = -1;
    bool finite = true;
    KernelTimer timer(b->stream, GAFIME_KERNEL_FINITE_CHECK);
    return check_finite(*b, &finite);
}

int gafime_contiguous_bucket_upload_columns(ContiguousBucket bucket, const float* h_cols, int64_t c0, int64_t c1,
                                            const float* h_y, const uint8_t* h_mask) {
    if (!bucket || !h_y || !h_mask) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    if (c0 < 0 || c1 < c0 || c1 > b->f || (c1 > c0 && !h_cols)) return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(b->device);
    // queued on the bucket's stream, where a collective that fills the other features runs
    cudaError_t e = cudaSuccess;
    if (c1 > c0)
        e = cudaMemcpy2DAsync(b->d_data + c0 * b->ld, (size_t)b->ld * sizeof(float), h_cols,
                              (size_t)b->n * sizeof(float), (size_t)b->n * sizeof(float), (size_t)(c1 - c0),
                              cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(b->d_data + b->f * b->ld, h_y, (size_t)b->n * sizeof(float), cudaMemcpyHostToDevice,
                            b->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b->d_mask, h_mask, (size_t)b->n, cudaMemcpyHostToDevice, b->stream);
    b->finite_state = -1;   // checked by the next scoring call
    return e == cudaSuccess ? GAFIME_SUCCESS : status_from(e);
}

int gafime_contiguous_bucket_device_columns(ContiguousBucket bucket, int64_t c0, int64_t c1, float** d_ptr,
                                            int64_t* ld) {
    if (!bucket || !d_ptr || !ld) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    if (c0 < 0 || c1 < c0 || c1 > b->f) return GAFIME_ERROR_INVALID_ARGS;
    *d_ptr = b->d_data + c0 * b->ld;
    *ld = b->ld;
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_mark_updated(ContiguousBucket bucket) {
    if (!bucket) return GAFIME_ERROR_INVALID_ARGS;
    ((Bucket*)bucket)->finite_state = -1;
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_upload_rows(ContiguousBucket bucket, const float* h_rows, const float* h_y,
                                         const uint8_t* h_mask) {
    if (!bucket || !h_rows || !h_y || !h_mask) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    cudaSetDevice(b->device);
    const int64_t f = b->f, n = b->n, ld = b->ld;
    // row chunks of at most 64 MB through two staging buffers: the copy of one chunk overlaps
    // the transpose of the previous one
    const int64_t chunk = std::max<int64_t>(32, std::min<int64_t>(n, ((int64_t)16 << 20) / f) / 32 * 32);
    cudaError_t e = ensure(b->gather, 2 * (size_t)chunk * f * sizeof(float));
    if (e != cudaSuccess) return status_from(e);
    float* stage[2] = {(float*)b->gather.ptr, (float*)b->gather.ptr + chunk * f};
    cudaEvent_t done[2] = {nullptr, nullptr};
    for (int s = 0; s < 2 && e == cudaSuccess; ++s) e = cudaEventCreateWithFlags(&done[s], cudaEventDisableTiming);
    int q = 0;
    for (int64_t r0 = 0; r0 < n && e == cudaSuccess; r0 += chunk, q ^= 1) {
        const int64_t rows = std::min<int64_t>(chunk, n - r0);
        // the staging buffer's previous transpose must be done before it is overwritten
        e = cudaEventSynchronize(done[q]);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(stage[q], h_rows + r0 * f, (size_t)rows * f * sizeof(float), cudaMemcpyHostToDevice,
                                b->stream);
        if (e != cudaSuccess) break;
        dim3 grid((unsigned)((f + 31) / 32), (unsigned)((rows + 31) / 32));
        rows_to_columns_kernel<<<grid, 256, 0, b->stream>>>(stage[q], rows, f, b->d_data, ld, r0);
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaEventRecord(done[q], b->stream);
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(b->d_data + f * ld, h_y, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b->d_mask, h_mask, (size_t)n, cudaMemcpyHostToDevice, b->stream);
    {
        // also after a failure: no copy from the caller's buffers is left in flight
        const cudaError_t es = cudaStreamSynchronize(b->stream);
        if (e == cudaSuccess) e = es;
    }
    for (int s = 0; s < 2; ++s)
        if (done[s]) cudaEventDestroy(done[s]);
    if (e != cudaSuccess) return status_from(e);
    b->finite_state = -1;
    bool finite = true;
    KernelTimer timer(b->stream, GAFIME_KERNEL_FINITE_CHECK);
    return check_finite(*b, &finite);
}

int gafime_contiguous_bucket_upload_target(ContiguousBucket bucket, const float* h_y) {
    if (!bucket || !h_y) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    cudaSetDevice(b->device);
    float* y = b->d_data + b->f * b->ld;
    cudaError_t e = cudaMemcpyAsync(y, h_y, (size_t)b->n * sizeof(float), cudaMemcpyHostToDevice, b->stream);
    if (e != cudaSuccess) return status_from(e);
    // features already known finite: only the new target needs the check
    const int features_finite = b->finite_state;
    b->finite_state = -1;
    if (features_finite != 1) {
        bool finite = true;
        return check_finite(*b, &finite);
    }
    e = ensure(b->flags, 64);
    int h = 0;
    if (e == cudaSuccess) e = cudaMemsetAsync((int*)b->flags.ptr, 0, sizeof(int), b->stream);
    if (e == cudaSuccess) {
        KernelTimer timer(b->stream, GAFIME_KERNEL_FINITE_CHECK);
        finite4_kernel<<<b->sm_count, 256, 0, b->stream>>>((const float4*)y, b->ld / 4, (int*)b->flags.ptr);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, b->flags.ptr, sizeof(int), cudaMemcpyDeviceToHost, b->stream);
    {
        // also after a failure: the copy of h_y is not left in flight
        const cudaError_t es = cudaStreamSynchronize(b->stream);
        if (e == cudaSuccess) e = es;
    }
    if (e != cudaSuccess) return status_from(e);
    b->finite_state = h == 0 ? 1 : 0;
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_gather(ContiguousBucket dst, ContiguousBucket src, const int32_t* cols,
                                    int32_t n_cols, const int64_t* rows, int64_t n_rows) {
    if (!dst || !src || dst == src || !cols) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* d = (Bucket*)dst;
    Bucket* s = (Bucket*)src;
    if (d->device != s->device || n_cols != d->f || n_rows != d->n || (!rows && n_rows != s->n))
        return GAFIME_ERROR_INVALID_ARGS;
    for (int32_t c = 0; c < n_cols; ++c)
        if (cols[c] < 0 || cols[c] >= s->f) return GAFIME_ERROR_INVALID_ARGS;
    if (rows)
        for (int64_t r = 0; r < n_rows; ++r)
            if (rows[r] < 0 || rows[r] >= s->n) return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(d->device);
    // source columns (the target last) and row indices, staged in dst's scratch
    const size_t col_bytes = ((size_t)(n_cols + 1) * sizeof(int32_t) + 255) / 256 * 256;
    const size_t row_bytes = rows ? (size_t)n_rows * sizeof(int64_t) : 0;
    cudaError_t e = ensure(d->gather, col_bytes + row_bytes);
    if (e != cudaSuccess) return status_from(e);
    std::vector<int32_t> scol(cols, cols + n_cols);
    scol.push_back((int32_t)s->f);
    int32_t* d_cols = (int32_t*)d->gather.ptr;
    int64_t* d_rows = rows ? (int64_t*)((char*)d->gather.ptr + col_bytes) : nullptr;
    // the source bucket's queued work (its upload) must finish before dst's stream reads it
    e = cudaStreamSynchronize(s->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_cols, scol.data(), scol.size() * sizeof(int32_t), cudaMemcpyHostToDevice, d->stream);
    if (e == cudaSuccess && rows)
        e = cudaMemcpyAsync(d_rows, rows, row_bytes, cudaMemcpyHostToDevice, d->stream);
    if (e != cudaSuccess) return status_from(e);
    // about 4 CTAs per SM: one grid row per destination column, enough row blocks to fill
    const int64_t cols_total = (int64_t)n_cols + 1, gy = std::min<int64_t>(cols_total, 65535);
    const int64_t gx = std::max<int64_t>(1, std::min<int64_t>((n_rows + 255) / 256, (4 * d->sm_count + gy - 1) / gy));
    dim3 grid((unsigned)gx, (unsigned)gy);
    gather_rows_kernel<<<grid, 256, 0, d->stream>>>(s->d_data, s->ld, d_cols, cols_total, d_rows, n_rows, d->d_data,
                                                    d->ld);
    gather_mask_kernel<<<(unsigned)std::min<int64_t>((n_rows + 255) / 256, 4 * d->sm_count), 256, 0, d->stream>>>(
        s->d_mask, d_rows, n_rows, d->d_mask);
    e = cudaGetLastError();
    {
        // also after a failure: the copy of the caller's row ids is not left in flight
        const cudaError_t es = cudaStreamSynchronize(d->stream);
        if (e == cudaSuccess) e = es;
    }
    if (e != cudaSuccess) return status_from(e);
    // rows of finite data are finite; anything else is checked like an upload
    d->finite_state = s->finite_state == 1 ? 1 : -1;
    bool finite = true;
    return check_finite(*d, &finite);
}

int gafime_contiguous_bucket_compute(ContiguousBucket bucket, int feature_a_idx, int feature_b_idx,
                                     int op_a, int op_b, int interact_type, int val_fold_id,
                                     float* h_stats_out) {
    if (!bucket || !h_stats_out) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    if (feature_a_idx < 0 || feature_a_idx >= b->f || feature_b_idx < 0 || feature_b_idx >= b->f)
        return GAFIME_ERROR_INVALID_ARGS;
    if (op_a < 0 || op_a > GAFIME_OP_ROLLING_STD || op_b < 0 || op_b > GAFIME_OP_ROLLING_STD ||
        interact_type < 0 || interact_type > GAFIME_INTERACT_MIN)
        return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(b->device);
    cudaError_t e = ensure(b->stats_part, (size_t)(kLegacyBlocks + 1) * 12 * sizeof(double));
    if (e != cudaSuccess) return status_from(e);
    double* part = (double*)b->stats_part.ptr;
    double* total = part + kLegacyBlocks * 12;
    KernelTimer timer(b->stream, GAFIME_KERNEL_LEGACY_PAIR);
    legacy_pair_stats_kernel<<<kLegacyBlocks, 256, 0, b->stream>>>(
        b->d_data, b->d_mask, b->n, b->ld, b->f, feature_a_idx, feature_b_idx, op_a, op_b,
        interact_type, val_fold_id, part);
    sum_partials_kernel<<<1, 32, 0, b->stream>>>(part, kLegacyBlocks, 12, total);
    e = cudaGetLastError();
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(b->h_pinned, total, 12 * sizeof(double), cudaMemcpyDeviceToHost,
                            b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return status_from(e);
    for (int m = 0; m < 12; ++m) h_stats_out[m] = (float)b->h_pinned[m];
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_free(ContiguousBucket bucket) {
    if (!bucket) return GAFIME_SUCCESS;
    Bucket* b = (Bucket*)bucket;
    cudaSetDevice(b->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    DeviceBuf* bufs[] = {&b->stats_part, &b->stats, &b->ycen, &b->xcen, &b->moments, &b->cands,
                         &b->cands2, &b->scores, &b->flags, &b->tiles, &b->mi, &b->mi_hist, &b->mi_mm, &b->mi_xs, &b->mi_split, &b->gather, &b->rank, &b->gram_cols,
                         &b->gram, &b->gram_planes, &b->guard};
    for (DeviceBuf* d : bufs) release(*d);
    if (b->d_data) cudaFree(b->d_data);
    if (b->d_mask) cudaFree(b->d_mask);
    if (b->h_pinned) cudaFreeHost(b->h_pinned);
    for (cudaEvent_t ev : b->arrived) cudaEventDestroy(ev);
    if (b->copy_stream) {
        cudaStreamSynchronize(b->copy_stream);
        cudaStreamDestroy(b->copy_stream);
    }
    if (b->stream) cudaStreamDestroy(b->stream);
    delete b;
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_stream(ContiguousBucket bucket, void** stream_out) {
    if (!bucket || !stream_out) return GAFIME_ERROR_INVALID_ARGS;
    *stream_out = (void*)((Bucket*)bucket)->stream;
    return GAFIME_SUCCESS;
}

int gafime_contiguous_bucket_info(ContiguousBucket bucket, int* n_samples_out, int* n_features_out) {
    if (!bucket) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    if (n_samples_out) *n_samples_out = (int)b->n;
    if (n_features_out) *n_features_out = (int)b->f;
    return GAFIME_SUCCESS;
}

}  // extern "C"

// ============================================================ GafimeBucket ABI ==
//
// The reference's small-bucket API (interfaces.h:176-382; GafimeBucketImpl and kernels in
// src/cuda/kernels.cu:589-1400), used by StaticBucket / FusedKernelWrapper
// (gafime/backends/fused_kernel.py:318-848): at most 5 feature columns, arity-2..5 chains
// x = combine(...combine(combine(op0(f0), op1(f1), t0), op2(f2), t1)..., t_{a-2}) in fp32
// (the per-pair-type form of cpu_backend.cpp:229-310), 12 stats split by fold.  Here the
// bucket is the contiguous bucket with F <= 5 (same column-major layout, y in column F);
// sums are fp64 in a fixed order and cast to float at the end, like the CPU reference.

namespace gafime {
namespace {

constexpr int kMaxChain = 5;       // GAFIME_MAX_FEATURES of the reference
constexpr int kMaxBatch = 1024;    // GAFIME_MAX_BATCH_SIZE of the reference

struct ChainDesc {
    int arity;
    int feat[kMaxChain];
    int op[kMaxChain];
    int inter[kMaxChain - 1];
};

__device__ __forceinline__ float chain_value(const float* __restrict__ data, int64_t ld, int64_t r,
                                             const ChainDesc& d) {
    float x = combine_op(apply_op(data[(int64_t)d.feat[0] * ld + r], d.op[0]),
                         apply_op(data[(int64_t)d.feat[1] * ld + r], d.op[1]), d.inter[0]);
    #pragma unroll
    for (int k = 2; k < kMaxChain; ++k)
        if (k < d.arity) x = combine_op(x, apply_op(data[(int64_t)d.feat[k] * ld + r], d.op[k]), d.inter[k - 1]);
    return x;
}

// Fixed-order reduction of NV doubles per thread over the block (256 threads): warp
// shuffles, then warps in order.  Result valid in thread 0.
template <int NV>
__device__ __forceinline__ void block_reduce_warps(double (&v)[NV], double* smem /*[8*NV]*/) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    #pragma unroll
    for (int m = 0; m < NV; ++m)
        for (int o = 16; o > 0; o >>= 1) v[m] += __shfl_down_sync(0xffffffffu, v[m], o);
    if (lane == 0)
        #pragma unroll
        for (int m = 0; m < NV; ++m) smem[warp * NV + m] = v[m];
    __syncthreads();
    if (threadIdx.x == 0)
        #pragma unroll
        for (int m = 0; m < NV; ++m) {
            double s = smem[m];
            for (int w = 1; w < 8; ++w) s += smem[w * NV + m];
            v[m] = s;
        }
}

// Grid (blocks, items): kSlots chains per item evaluated on the same rows.  A row is
// skipped when y or any slot's x is NaN (with two slots this is the interleaved kernel's
// rule, kernels.cu:1217-1218).
template <int kSlots>
__global__ void __launch_bounds__(256) chain_stats_kernel(const float* __restrict__ data,
                                                          const uint8_t* __restrict__ mask, int64_t n,
                                                          int64_t ld, int64_t ycol,
                                                          const ChainDesc* __restrict__ descs, int val_fold_id,
                                                          double* __restrict__ partial) {
    __shared__ double red[8 * 12 * kSlots];
    ChainDesc d[kSlots];
    #pragma unroll
    for (int s = 0; s < kSlots; ++s) d[s] = descs[blockIdx.y * kSlots + s];
    double acc[12 * kSlots];
    #pragma unroll
    for (int m = 0; m < 12 * kSlots; ++m) acc[m] = 0.0;
    const float* y = data + ycol * ld;
    for (int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x; r < n; r += (int64_t)gridDim.x * 256) {
        float x[kSlots];
        bool skip = false;
        #pragma unroll
        for (int s = 0; s < kSlots; ++s) {
            x[s] = chain_value(data, ld, r, d[s]);
            skip |= isnan(x[s]);
        }
        const float yv = y[r];
        if (skip || isnan(yv)) continue;
        const int o = (mask[r] == val_fold_id) ? 6 : 0;
        const double yd = yv;
        #pragma unroll
        for (int s = 0; s < kSlots; ++s) {
            const double xd = x[s];
            #pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (o == 6 * h) {
                    double* a = acc + 12 * s + 6 * h;
                    a[0] += 1.0;
                    a[1] += xd;
                    a[2] += yd;
                    a[3] += xd * xd;
                    a[4] += yd * yd;
                    a[5] += xd * yd;
                }
            }
        }
    }
    block_reduce_warps<12 * kSlots>(acc, red);
    if (threadIdx.x == 0) {
        double* out = partial + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * 12 * kSlots;
        #pragma unroll
        for (int m = 0; m < 12 * kSlots; ++m) out[m] = acc[m];
    }
}

// out[item][m] = sum over the blocks of partial[item][block][m], in block order
__global__ void sum_item_partials_kernel(const double* __restrict__ partial, int blocks, int width,
                                         double* __restrict__ out) {
    const int item = blockIdx.x, m = threadIdx.x;
    if (m >= width) return;
    double s = 0.0;
    for (int b = 0; b < blocks; ++b) s += partial[((int64_t)item * blocks + b) * width + m];
    out[(int64_t)item * width + m] = s;
}

bool valid_unary(int op) { return op >= GAFIME_OP_IDENTITY && op <= GAFIME_OP_ROLLING_STD; }
bool valid_combiner(int t) { return t >= GAFIME_INTERACT_MULT && t <= GAFIME_INTERACT_MIN; }

// Row blocks per item of the chain kernel: about four CTAs per SM over all items.
int chain_blocks(const Bucket& b, int items) {
    int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((b.n + 255) / 256, (4 * (int64_t)b.sm_count + items - 1) / items));
    return std::min(blocks, 1024);
}

// Queue the chain kernel and the per-item sums on `stream`: d_out[items][12 * kSlots].
template <int kSlots>
cudaError_t launch_chains(const Bucket& b, const ChainDesc* d_descs, int items, int val_fold_id, double* d_part,
                          double* d_out, cudaStream_t stream) {
    const int blocks = chain_blocks(b, items);
    chain_stats_kernel<kSlots><<<dim3((unsigned)blocks, (unsigned)items), 256, 0, stream>>>(
        b.d_data, b.d_mask, b.n, b.ld, b.f, d_descs, val_fold_id, d_part);
    sum_item_partials_kernel<<<items, 32, 0, stream>>>(d_part, blocks, 12 * kSlots, d_out);
    return cudaGetLastError();
}

// Run `items` chain groups of kSlots chains and write items x (12 * kSlots) float stats.
template <int kSlots>
int run_chains(Bucket& b, const ChainDesc* h_descs, int items, int val_fold_id, float* h_stats) {
    const int width = 12 * kSlots;
    const int blocks = chain_blocks(b, items);
    const size_t desc_bytes = (size_t)items * kSlots * sizeof(ChainDesc);
    const size_t part_bytes = (size_t)items * blocks * width * sizeof(double);
    const size_t off_part = (desc_bytes + 255) / 256 * 256;
    const size_t off_out = (off_part + part_bytes + 255) / 256 * 256;
    const size_t out_bytes = (size_t)items * width * sizeof(double);
    cudaError_t e = ensure(b.stats_part, off_out + out_bytes);
    if (e != cudaSuccess) return status_from(e);
    char* base = (char*)b.stats_part.ptr;
    ChainDesc* d_descs = (ChainDesc*)base;
    double* d_part = (double*)(base + off_part);
    double* d_out = (double*)(base + off_out);
    std::vector<double> host((size_t)items * width);
    e = cudaMemcpyAsync(d_descs, h_descs, desc_bytes, cudaMemcpyHostToDevice, b.stream);
    if (e == cudaSuccess) {
        KernelTimer timer(b.stream, GAFIME_KERNEL_LEGACY_PAIR);
        e = launch_chains<kSlots>(b, d_descs, items, val_fold_id, d_part, d_out, b.stream);
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(host.data(), d_out, out_bytes, cudaMemcpyDeviceToHost, b.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b.stream);
    if (e != cudaSuccess) return status_from(e);
    for (size_t m = 0; m < host.size(); ++m) h_stats[m] = (float)host[m];
    return GAFIME_SUCCESS;
}

int upload_column(Bucket* b, int64_t col, const void* h, size_t bytes) {
    cudaSetDevice(b->device);
    cudaError_t e = cudaMemcpyAsync(b->d_data + col * b->ld, h, bytes, cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    b->finite_state = -1;
    return e == cudaSuccess ? GAFIME_SUCCESS : GAFIME_ERROR_KERNEL_FAILED;
}

}  // namespace
}  // namespace gafime

namespace gafime {
namespace {
// Arity-2 descriptors of a batch (indices / ops [2 per item], one combiner per item);
// false when an id is out of range.
bool batch_descs(const Bucket& b, const int* idx, const int* ops, const int* inter, int n, ChainDesc* d) {
    for (int q = 0; q < n; ++q) {
        ChainDesc& c = d[q];
        c = ChainDesc{};
        c.arity = 2;
        for (int k = 0; k < 2; ++k) {
            const int fi = idx[2 * q + k], op = ops[2 * q + k];
            if (fi < 0 || fi >= b.f || !valid_unary(op)) return false;
            c.feat[k] = fi;
            c.op[k] = op;
        }
        if (!valid_combiner(inter[q])) return false;
        c.inter[0] = inter[q];
    }
    return true;
}
}  // namespace
}  // namespace gafime

extern "C" int gafime_bucket_alloc(int n_samples, int n_features, GafimeBucket* bucket_out) {
    if (n_samples <= 0 || n_features <= 0 || n_features > kMaxChain || !bucket_out) return GAFIME_ERROR_INVALID_ARGS;
    return gafime_contiguous_bucket_alloc(n_samples, n_features, (ContiguousBucket*)bucket_out);
}

extern "C" int gafime_bucket_upload_feature(GafimeBucket bucket, int feature_idx, const float* h_data) {
    if (!bucket || !h_data) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    if (feature_idx < 0 || feature_idx >= b->f) return GAFIME_ERROR_INVALID_ARGS;
    return upload_column(b, feature_idx, h_data, (size_t)b->n * sizeof(float));
}

extern "C" int gafime_bucket_upload_target(GafimeBucket bucket, const float* h_target) {
    if (!bucket || !h_target) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    return upload_column(b, b->f, h_target, (size_t)b->n * sizeof(float));
}

extern "C" int gafime_bucket_upload_mask(GafimeBucket bucket, const uint8_t* h_mask) {
    if (!bucket || !h_mask) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    cudaSetDevice(b->device);
    cudaError_t e = cudaMemcpyAsync(b->d_mask, h_mask, (size_t)b->n, cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    return e == cudaSuccess ? GAFIME_SUCCESS : GAFIME_ERROR_KERNEL_FAILED;
}

extern "C" int gafime_bucket_compute(GafimeBucket bucket, const int* feature_indices, const int* ops, int arity,
                                     const int* interaction_types, int val_fold_id, float* h_stats) {
    if (!bucket || !feature_indices || !ops || !interaction_types || !h_stats) return GAFIME_ERROR_INVALID_ARGS;
    if (arity < 2 || arity > kMaxChain) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    ChainDesc d{};
    d.arity = arity;
    for (int k = 0; k < arity; ++k) {
        if (feature_indices[k] < 0 || feature_indices[k] >= b->f || !valid_unary(ops[k])) return GAFIME_ERROR_INVALID_ARGS;
        d.feat[k] = feature_indices[k];
        d.op[k] = ops[k];
        if (k > 0) {
            if (!valid_combiner(interaction_types[k - 1])) return GAFIME_ERROR_INVALID_ARGS;
            d.inter[k - 1] = interaction_types[k - 1];
        }
    }
    cudaSetDevice(b->device);
    return run_chains<1>(*b, &d, 1, val_fold_id, h_stats);
}

extern "C" int gafime_bucket_compute_batch(GafimeBucket bucket, const int* batch_indices, const int* batch_ops,
                                           const int* batch_interact, int batch_size, int val_fold_id,
                                           float* h_stats_batch) {
    if (!bucket || !batch_indices || !batch_ops || !batch_interact || !h_stats_batch) return GAFIME_ERROR_INVALID_ARGS;
    if (batch_size <= 0 || batch_size > kMaxBatch) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    std::vector<ChainDesc> d((size_t)batch_size);
    if (!batch_descs(*b, batch_indices, batch_ops, batch_interact, batch_size, d.data()))
        return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(b->device);
    return run_chains<1>(*b, d.data(), batch_size, val_fold_id, h_stats_batch);
}

extern "C" int gafime_interleaved_compute(GafimeBucket bucket, const int* feature_indices_A, const int* ops_A,
                                          int arity_A, int interact_A, const int* feature_indices_B,
                                          const int* ops_B, int arity_B, int interact_B, int window_size,
                                          int val_fold_id, float* h_stats_A, float* h_stats_B) {
    (void)window_size;   // rolling operators evaluate to NaN on the device, as in the reference
    if (!bucket || !feature_indices_A || !ops_A || !feature_indices_B || !ops_B || !h_stats_A || !h_stats_B)
        return GAFIME_ERROR_INVALID_ARGS;
    if (arity_A != 2 || arity_B != 2) return GAFIME_ERROR_INVALID_ARGS;   // kernels.cu:1348-1351
    Bucket* b = (Bucket*)bucket;
    ChainDesc d[2] = {};
    const int* fi[2] = {feature_indices_A, feature_indices_B};
    const int* op[2] = {ops_A, ops_B};
    const int it[2] = {interact_A, interact_B};
    for (int s = 0; s < 2; ++s) {
        d[s].arity = 2;
        for (int k = 0; k < 2; ++k) {
            if (fi[s][k] < 0 || fi[s][k] >= b->f || !valid_unary(op[s][k])) return GAFIME_ERROR_INVALID_ARGS;
            d[s].feat[k] = fi[s][k];
            d[s].op[k] = op[s][k];
        }
        if (!valid_combiner(it[s])) return GAFIME_ERROR_INVALID_ARGS;
        d[s].inter[0] = it[s];
    }
    cudaSetDevice(b->device);
    float both[24];
    const int st = run_chains<2>(*b, d, 1, val_fold_id, both);
    if (st != GAFIME_SUCCESS) return st;
    for (int m = 0; m < 12; ++m) {
        h_stats_A[m] = both[m];
        h_stats_B[m] = both[12 + m];
    }
    return GAFIME_SUCCESS;
}

extern "C" int gafime_bucket_free(GafimeBucket bucket) { return gafime_contiguous_bucket_free((ContiguousBucket)bucket); }

// Legacy one-shot form (interfaces.h:372-382): a temporary bucket per call, one interaction
// type for every step of the chain (gafime_fused_interaction_cpu, cpu_backend.cpp:127-213).
extern "C" int gafime_fused_interaction(const float** h_inputs, const float* h_target, const uint8_t* h_mask,
                                        const int* h_ops, int arity, int interaction_type, int val_fold_id,
                                        int n_samples, float* h_stats) {
    if (!h_inputs || !h_target || !h_mask || !h_ops || !h_stats) return GAFIME_ERROR_INVALID_ARGS;
    if (arity < 2 || arity > kMaxChain || n_samples <= 0) return GAFIME_ERROR_INVALID_ARGS;
    for (int k = 0; k < arity; ++k)
        if (!h_inputs[k] || !valid_unary(h_ops[k])) return GAFIME_ERROR_INVALID_ARGS;
    if (!valid_combiner(interaction_type)) return GAFIME_ERROR_INVALID_ARGS;
    GafimeBucket b = nullptr;
    int st = gafime_bucket_alloc(n_samples, arity, &b);
    if (st != GAFIME_SUCCESS) return st;
    for (int k = 0; k < arity && st == GAFIME_SUCCESS; ++k) st = gafime_bucket_upload_feature(b, k, h_inputs[k]);
    if (st == GAFIME_SUCCESS) st = gafime_bucket_upload_target(b, h_target);
    if (st == GAFIME_SUCCESS) st = gafime_bucket_upload_mask(b, h_mask);
    if (st == GAFIME_SUCCESS) {
        int fi[kMaxChain], types[kMaxChain - 1];
        for (int k = 0; k < arity; ++k) fi[k] = k;
        for (int k = 0; k + 1 < arity; ++k) types[k] = interaction_type;
        st = gafime_bucket_compute(b, fi, h_ops, arity, types, val_fold_id, h_stats);
    }
    gafime_bucket_free(b);
    return st;
}

// ============================================================ async pipeline ==
//
// The reference's 4-slot ring (interfaces.h:433-504, kernels.cu:1755-2140): submit queues a
// batch of arity-2 interactions on its slot's stream and returns at once (PIPELINE_FULL when
// four batches are in flight); poll / wait hand back the oldest batch first; flush drains
// every pending batch in submission order.  Each slot owns pinned staging and device
// buffers sized for the largest batch, so submit allocates nothing.

namespace gafime {
namespace {

constexpr int kPipeSlots = 4;      // PIPELINE_SLOTS
constexpr int kPipeMaxBatch = 1024; // PIPELINE_MAX_BATCH

struct PipeSlot {
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    ChainDesc* h_desc = nullptr;   // pinned [kPipeMaxBatch]
    double* h_out = nullptr;       // pinned [kPipeMaxBatch * 12]
    ChainDesc* d_desc = nullptr;
    double* d_part = nullptr;      // [kPipeMaxBatch * max blocks * 12]
    double* d_out = nullptr;       // [kPipeMaxBatch * 12]
    int batch = 0;
    bool busy = false;
};

struct Pipeline {
    Bucket* b = nullptr;
    int val_fold = 0;
    PipeSlot slots[kPipeSlots];
    int read = 0, write = 0, pending = 0;
};

void pipe_release(Pipeline* p) {
    for (PipeSlot& s : p->slots) {
        if (s.done) cudaEventSynchronize(s.done);
        if (s.stream) cudaStreamDestroy(s.stream);
        if (s.done) cudaEventDestroy(s.done);
        if (s.h_desc) cudaFreeHost(s.h_desc);
        if (s.h_out) cudaFreeHost(s.h_out);
        if (s.d_desc) cudaFree(s.d_desc);
        if (s.d_part) cudaFree(s.d_part);
        if (s.d_out) cudaFree(s.d_out);
    }
    delete p;
}

// hand the oldest batch back (its event has completed)
void pipe_pop(Pipeline* p, float* h_stats_out, int* batch_size_out) {
    PipeSlot& s = p->slots[p->read];
    if (h_stats_out)
        for (int m = 0; m < s.batch * 12; ++m) h_stats_out[m] = (float)s.h_out[m];
    if (batch_size_out) *batch_size_out = s.batch;
    s.batch = 0;
    s.busy = false;
    p->read = (p->read + 1) % kPipeSlots;
    --p->pending;
}

}  // namespace
}  // namespace gafime

extern "C" int gafime_pipeline_init(GafimeBucket bucket, int val_fold_id, GafimePipeline* pipeline_out) {
    if (!bucket || !pipeline_out) return GAFIME_ERROR_INVALID_ARGS;
    Bucket* b = (Bucket*)bucket;
    cudaSetDevice(b->device);
    Pipeline* p = new (std::nothrow) Pipeline();
    if (!p) return GAFIME_ERROR_OUT_OF_MEMORY;
    p->b = b;
    p->val_fold = val_fold_id;
    int max_part = 0;
    for (int items = 1; items <= kPipeMaxBatch; ++items) max_part = std::max(max_part, items * chain_blocks(*b, items));
    cudaError_t e = cudaSuccess;
    for (PipeSlot& s : p->slots) {
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaMallocHost(&s.h_desc, kPipeMaxBatch * sizeof(ChainDesc));
        if (e == cudaSuccess) e = cudaMallocHost(&s.h_out, kPipeMaxBatch * 12 * sizeof(double));
        if (e == cudaSuccess) e = cudaMalloc(&s.d_desc, kPipeMaxBatch * sizeof(ChainDesc));
        if (e == cudaSuccess) e = cudaMalloc(&s.d_part, (size_t)max_part * 12 * sizeof(double));
        if (e == cudaSuccess) e = cudaMalloc(&s.d_out, kPipeMaxBatch * 12 * sizeof(double));
    }
    if (e != cudaSuccess) {
        pipe_release(p);
        cudaGetLastError();
        return e == cudaErrorMemoryAllocation ? GAFIME_ERROR_OUT_OF_MEMORY : GAFIME_ERROR_KERNEL_FAILED;
    }
    *pipeline_out = p;
    return GAFIME_SUCCESS;
}

extern "C" int gafime_pipeline_submit(GafimePipeline pipeline, const int* h_indices, const int* h_ops,
                                      const int* h_interact, int batch_size, int* slot_id_out) {
    if (!pipeline || !h_indices || !h_ops || !h_interact) return GAFIME_ERROR_INVALID_ARGS;
    if (batch_size <= 0 || batch_size > kPipeMaxBatch) return GAFIME_ERROR_INVALID_ARGS;
    Pipeline* p = (Pipeline*)pipeline;
    if (p->pending >= kPipeSlots) {
        if (slot_id_out) *slot_id_out = -1;
        return GAFIME_ERROR_PIPELINE_FULL;
    }
    const int id = p->write;
    PipeSlot& s = p->slots[id];
    if (!batch_descs(*p->b, h_indices, h_ops, h_interact, batch_size, s.h_desc)) return GAFIME_ERROR_INVALID_ARGS;
    cudaSetDevice(p->b->device);
    cudaError_t e = cudaMemcpyAsync(s.d_desc, s.h_desc, (size_t)batch_size * sizeof(ChainDesc), cudaMemcpyHostToDevice,
                                    s.stream);
    if (e == cudaSuccess) e = launch_chains<1>(*p->b, s.d_desc, batch_size, p->val_fold, s.d_part, s.d_out, s.stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(s.h_out, s.d_out, (size_t)batch_size * 12 * sizeof(double), cudaMemcpyDeviceToHost, s.stream);
    if (e == cudaSuccess) e = cudaEventRecord(s.done, s.stream);
    if (e != cudaSuccess) return GAFIME_ERROR_KERNEL_FAILED;
    s.batch = batch_size;
    s.busy = true;
    p->write = (p->write + 1) % kPipeSlots;
    ++p->pending;
    if (slot_id_out) *slot_id_out = id;
    return GAFIME_SUCCESS;
}

extern "C" int gafime_pipeline_poll(GafimePipeline pipeline, float* h_stats_out, int* batch_size_out) {
    if (!pipeline) return GAFIME_ERROR_INVALID_ARGS;
    Pipeline* p = (Pipeline*)pipeline;
    if (p->pending == 0) return GAFIME_ERROR_NO_RESULT;
    const cudaError_t e = cudaEventQuery(p->slots[p->read].done);
    if (e == cudaErrorNotReady) return GAFIME_ERROR_NO_RESULT;
    if (e != cudaSuccess) return GAFIME_ERROR_KERNEL_FAILED;
    pipe_pop(p, h_stats_out, batch_size_out);
    return GAFIME_SUCCESS;
}

extern "C" int gafime_pipeline_wait(GafimePipeline pipeline, float* h_stats_out, int* batch_size_out) {
    if (!pipeline) return GAFIME_ERROR_INVALID_ARGS;
    Pipeline* p = (Pipeline*)pipeline;
    if (p->pending == 0) return GAFIME_ERROR_NO_RESULT;
    if (cudaEventSynchronize(p->slots[p->read].done) != cudaSuccess) return GAFIME_ERROR_KERNEL_FAILED;
    pipe_pop(p, h_stats_out, batch_size_out);
    return GAFIME_SUCCESS;
}

extern "C" int gafime_pipeline_pending(GafimePipeline pipeline) {
    return pipeline ? ((Pipeline*)pipeline)->pending : 0;
}

extern "C" int gafime_pipeline_flush(GafimePipeline pipeline, float* h_all_stats_out, int* total_batch_size_out) {
    if (!pipeline) return GAFIME_ERROR_INVALID_ARGS;
    Pipeline* p = (Pipeline*)pipeline;
    int total = 0;
    float* w = h_all_stats_out;
    while (p->pending > 0) {
        int n = 0;
        const int st = gafime_pipeline_wait(pipeline, w, &n);
        if (st != GAFIME_SUCCESS) return st;
        total += n;
        if (w) w += (size_t)n * 12;
    }
    if (total_batch_size_out) *total_batch_size_out = total;
    return GAFIME_SUCCESS;
}

extern "C" int gafime_pipeline_free(GafimePipeline pipeline) {
    if (!pipeline) return GAFIME_SUCCESS;
    Pipeline* p = (Pipeline*)pipeline;
    cudaSetDevice(p->b->device);
    pipe_release(p);
    return GAFIME_SUCCESS;
}
