// gram.cu -- pair moments as tcgen05 Gram tiles (sm_100a tensor cores).
//
// For a 128 x 128 block of column pairs (i in block I, j in block J) the three pair
// moments are dense contractions over rows:
//     C = sum a'b'            (centred columns a' = a - mean_a, b' = g(b) - mean_g)
//     Q = sum a^2 g(b)^2      (raw squares)
//     W = sum (a' ycen) b'    (ycen = y - mean y)
// with g = identity (multiply; add / subtract reuse C) or g(b) = 1/safe(b) (divide).
// They are computed by tcgen05.mma kind::f16 with fp32 accumulators in tensor memory
// (TMEM columns 0-127: C, 128-255: Q, 256-383: W).  Operands are fp16 planes stored row-major
// ([row][column], so a 16-row x 64-column TMA box is 16 runs of 128 B and the MMA reads
// MN-major operands), prepared once per call by gram_prep_kernel with every column scaled by
// a power of two so its largest magnitude is at most 2^14:
//     XH = fp16(s a'),  XL = fp16(s a' - XH)          (2-term split, ~22 bits)
//     QH/QL = 2-term split of s_q a^2
//     WH/WL = 2-term split of s_w a' ycen
//     GH/GL, GQH/GQL: the same for g(b) and g(b)^2 (divide only)
// Each Gram is hi.hi + hi.lo + lo.hi (the lo.lo term is below fp32 rounding): nine MMAs per
// 16-row step.  One fp16 term is not enough when a few rows dominate a sum (heavy tails,
// near-zero divisors): their 2^-12 rounding would not average out.
//
// Pipeline per CTA (one tile x one row chunk of <= 8192 rows, so each fp32 accumulation
// stays short): warp 0 issues TMA copies (2-D tensor maps, 128-byte swizzle, no multicast)
// of 10 operand tiles (two 64-column boxes each) per 16-row stage into a 5-stage ring; warp 1 issues the MMAs and
// commits each stage back to its "empty" barrier; warps 2-5 drain TMEM (tcgen05.ld) into
// fp32 partials [chunk][tile][C|Q|W][n][m] in HBM.  gram_reduce_kernel adds the chunks in
// fp64 in a fixed order, undoes the scales and the centring, and writes the raw moments
// S1 = sum a g(b), S2 = Q, S3 = sum a g(b) ycen that select.cu's epilogue scores.
//
// Every mbarrier wait is bounded: on timeout the thread records an error code in err[0],
// stops issuing work, drains what it issued, and the CTA frees its TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"

namespace gafime {

namespace {

constexpr int kGT = 128;                      // Gram tile edge (columns)
constexpr int kGK = 16;                       // rows per pipeline stage (one MMA K step)
constexpr int kGStages = 5;
constexpr int kOpBytes = kGT * kGK * 2;       // one operand tile: 128 columns x 16 rows fp16
constexpr int kNumA = 6, kNumB = 4;
constexpr int kStageBytes = (kNumA + kNumB) * kOpBytes;
constexpr int kGramThreads = 192;
constexpr uint32_t kTmemCols = 512;
constexpr long long kSpinLimit = 1LL << 24;
constexpr int64_t kMaxChunkRows = 8192;

enum Plane { P_XH = 0, P_XL, P_QH, P_QL, P_WH, P_WL, P_GH, P_GL, P_GQH, P_GQL, P_COUNT };

struct GramMaps {
    CUtensorMap m[P_COUNT];
};

struct GramArgs {
    const TileCoord* tiles;   // 128-blocks (bi, bj), bi <= bj
    int n_tiles;
    int64_t chunk_rows;       // multiple of kGK
    int64_t rows;             // padded rows (ld)
    int a_plane[kNumA];       // XH, XL, QH, QL, WH, WL
    int b_plane[kNumB];       // XH|GH, XL|GL, QH|GQH, QL|GQL
    float* partial;           // [chunk][tile][3][128 n][128 m]
    int* err;
};

// ---- PTX helpers ---------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase completed, false (error recorded) on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    for (long long i = 0; i < kSpinLimit; ++i)
        if (mbar_try(bar, parity)) return true;
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// MN-major operand tile, 128-byte swizzle: 64 columns (128 B) per swizzle row, 16 K rows;
// the two 64-column halves of a 128-column tile are 2048 B apart (LBO) and the two 8-row K
// groups 1024 B apart (SBO); descriptor version 1, layout code 2.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(2048 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32, A/B f16, both MN-major, N = 128, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | (1u << 15) | (1u << 16) |
                            ((uint32_t)(kGT >> 3) << 17) | ((uint32_t)(kGT >> 4) << 24);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    #pragma unroll
    for (int c = 0; c < 32; ++c) v[c] = __uint_as_float(r[c]);
}

// ---- the Gram kernel -------------------------------------------------------------

__global__ void __launch_bounds__(kGramThreads, 1)
gram_tile_kernel(const __grid_constant__ GramMaps maps, const GramArgs a) {
    extern __shared__ __align__(1024) unsigned char gsmem_raw[];
    // 1024-byte alignment for the swizzled tiles
    unsigned char* smem = (unsigned char*)(((uintptr_t)gsmem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + kGStages * kStageBytes);   // full[S], empty[S], accum
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kGStages + 1);
    const uint32_t smem0 = smem_u32(smem);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kGStages);
    const uint32_t accum = smem_u32(bars + 2 * kGStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileCoord tc = a.tiles[blockIdx.x];
    const int64_t r0 = (int64_t)blockIdx.y * a.chunk_rows;
    const int64_t r1 = min(r0 + a.chunk_rows, a.rows);
    const int nk = r1 > r0 ? (int)((r1 - r0) / kGK) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // producer: 10 operand tiles per stage
            int issued = 0;
            bool ok = true;
            for (int k = 0; k < nk && ok; ++k) {
                const int s = k % kGStages;
                if (k >= kGStages) ok = mbar_wait(empty0 + 8 * s, ((k / kGStages) - 1) & 1, a.err, 1);
                if (!ok) break;
                const uint32_t full = full0 + 8 * s;
                mbar_expect_tx(full, (uint32_t)kStageBytes);
                const uint32_t st = smem0 + s * kStageBytes;
                const int x = (int)(r0 + (int64_t)k * kGK);  // first row of the stage
                #pragma unroll
                for (int o = 0; o < kNumA; ++o)
                    #pragma unroll
                    for (int h = 0; h < 2; ++h)
                        tma_load_2d(st + o * kOpBytes + h * (kOpBytes / 2), &maps.m[a.a_plane[o]], full,
                                    tc.bi * kGT + h * 64, x);
                #pragma unroll
                for (int o = 0; o < kNumB; ++o)
                    #pragma unroll
                    for (int h = 0; h < 2; ++h)
                        tma_load_2d(st + (kNumA + o) * kOpBytes + h * (kOpBytes / 2), &maps.m[a.b_plane[o]],
                                    full, tc.bj * kGT + h * 64, x);
                ++issued;
            }
            if (!ok) {
                // drain: wait (bounded) for every stage that may still be filling
                for (int k = max(0, issued - kGStages); k < issued; ++k)
                    mbar_wait(full0 + 8 * (k % kGStages), (k / kGStages) & 1, a.err, 4);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer
            for (int k = 0; k < nk; ++k) {
                const int s = k % kGStages;
                if (!mbar_wait(full0 + 8 * s, (k / kGStages) & 1, a.err, 2)) break;
                tc_fence_after();
                const uint32_t st = smem0 + s * kStageBytes;
                const uint64_t aXH = umma_desc(st + 0 * kOpBytes), aXL = umma_desc(st + 1 * kOpBytes);
                const uint64_t aQH = umma_desc(st + 2 * kOpBytes), aQL = umma_desc(st + 3 * kOpBytes);
                const uint64_t aWH = umma_desc(st + 4 * kOpBytes), aWL = umma_desc(st + 5 * kOpBytes);
                const uint64_t bH = umma_desc(st + 6 * kOpBytes), bL = umma_desc(st + 7 * kOpBytes);
                const uint64_t bQH = umma_desc(st + 8 * kOpBytes), bQL = umma_desc(st + 9 * kOpBytes);
                const uint32_t acc = k > 0 ? 1u : 0u;
                umma(tmem + 0, aXH, bH, acc);      // C: hi x hi
                umma(tmem + 0, aXH, bL, 1u);       //    hi x lo
                umma(tmem + 0, aXL, bH, 1u);       //    lo x hi
                umma(tmem + 128, aQH, bQH, acc);   // Q
                umma(tmem + 128, aQH, bQL, 1u);
                umma(tmem + 128, aQL, bQH, 1u);
                umma(tmem + 256, aWH, bH, acc);    // W
                umma(tmem + 256, aWH, bL, 1u);
                umma(tmem + 256, aWL, bH, 1u);
                umma_commit(empty0 + 8 * s);  // stage free once these MMAs have read it
            }
            umma_commit(accum);  // all issued MMAs complete (also on the error path)
        }
    } else {
        // epilogue warps 2..5: TMEM lanes 32*(warp%4) .. +31 hold rows m of the tile.
        // The outcome is made warp-uniform: tcgen05.ld below is a whole-warp instruction.
        const bool ok = __all_sync(0xffffffffu, mbar_wait(accum, 0, a.err, 3));
        tc_fence_after();
        if (ok && nk > 0) {
            const int q = warp & 3;
            const int m = q * 32 + lane;
            float* out = a.partial + ((int64_t)blockIdx.y * a.n_tiles + blockIdx.x) * 3 * kGT * kGT;
            #pragma unroll 1
            for (int g = 0; g < 3; ++g) {
                #pragma unroll 1
                for (int c0 = 0; c0 < kGT; c0 += 32) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(g * kGT + c0), v);
                    float* o = out + (int64_t)g * kGT * kGT + (int64_t)c0 * kGT + m;
                    #pragma unroll
                    for (int c = 0; c < 32; ++c) o[(int64_t)c * kGT] = v[c];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        // no MMA may still be writing TMEM when it is freed (bounded, returns at once
        // when the accumulator barrier has already completed)
        if (lane == 0) mbar_wait(accum, 0, a.err, 5);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- operand preparation ------------------------------------------------------------

// Per column and row split: [0] min x, [1] max x, [2] sum g, [3] sum g^2, [4] sum g*ycen,
// [5] min g, [6] max g
struct GramColPart {
    double v[7];
};

__device__ __forceinline__ float safe_recip(float v, float eps) {
    float d = fabsf(v) < eps ? copysignf(eps, v) : v;
    return __frcp_rn(d);
}

__global__ void __launch_bounds__(256) gram_colstats_kernel(const float* __restrict__ x, int64_t ld, int64_t n,
                                                            const float* __restrict__ ycen, int recip,
                                                            float eps, int64_t span, GramColPart* part) {
    __shared__ double red[7][256];
    const int c = blockIdx.x, s = blockIdx.y, splits = gridDim.y;
    const int64_t rb = (int64_t)s * span, re = min(rb + span, n);
    double v[7] = {INFINITY, -INFINITY, 0.0, 0.0, 0.0, INFINITY, -INFINITY};
    for (int64_t r = rb + threadIdx.x; r < re; r += 256) {
        float xv = x[(int64_t)c * ld + r];
        v[0] = fmin(v[0], (double)xv);
        v[1] = fmax(v[1], (double)xv);
        if (recip) {
            double g = safe_recip(xv, eps);
            v[2] += g;
            v[3] += g * g;
            v[4] += g * (double)ycen[r];
            v[5] = fmin(v[5], g);
            v[6] = fmax(v[6], g);
        }
    }
    for (int m = 0; m < 7; ++m) red[m][threadIdx.x] = v[m];
    __syncthreads();
    for (int st = 128; st > 0; st >>= 1) {
        if (threadIdx.x < st) {
            int t = threadIdx.x;
            red[0][t] = fmin(red[0][t], red[0][t + st]);
            red[1][t] = fmax(red[1][t], red[1][t + st]);
            red[2][t] += red[2][t + st];
            red[3][t] += red[3][t + st];
            red[4][t] += red[4][t + st];
            red[5][t] = fmin(red[5][t], red[5][t + st]);
            red[6][t] = fmax(red[6][t], red[6][t + st]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        GramColPart p;
        for (int m = 0; m < 7; ++m) p.v[m] = red[m][0];
        part[(int64_t)c * splits + s] = p;
    }
}

// Per-column scales and statistics of the operands:
//   cs[c*12 + 0..4]: s_x, s_q, s_w, s_g, s_gq (powers of two)
//   cs[c*12 + 5]: mean g rounded to fp32 (the value the planes subtract)
//   cs[c*12 + 6..8]: sum g, sum g^2, sum g*ycen
//   cs[c*12 + 9]: mean x rounded to fp32 (the value the planes subtract)
struct GramScaleArgs {
    const GramColPart* part;
    int splits;
    int64_t f, n;
    const double* colstats;   // sum, sumsq, sum*ycen, mean per column
    double ycen_absmax;
    int recip;
    double* cs;
};

__device__ __forceinline__ double pow2_scale(double maxabs) {
    // largest power of two s with s * maxabs <= 2^14
    if (!(maxabs > 0.0) || !isfinite(maxabs)) return 1.0;
    int e;
    frexp(16384.0 / maxabs, &e);  // 16384/maxabs = f * 2^e, f in [0.5, 1)
    return ldexp(1.0, e - 1);
}

__global__ void gram_scale_kernel(GramScaleArgs a) {
    int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= a.f) return;
    double mn = INFINITY, mx = -INFINITY, sg = 0, sgg = 0, sgy = 0, gmn = INFINITY, gmx = -INFINITY;
    for (int s = 0; s < a.splits; ++s) {
        const GramColPart& p = a.part[c * a.splits + s];
        mn = fmin(mn, p.v[0]);
        mx = fmax(mx, p.v[1]);
        sg += p.v[2];
        sgg += p.v[3];
        sgy += p.v[4];
        gmn = fmin(gmn, p.v[5]);
        gmx = fmax(gmx, p.v[6]);
    }
    const double mu = (double)(float)a.colstats[c * 4 + 3];
    // the fp32 subtraction may round up by one ulp: a 2^-20 margin keeps |value| <= 2^14
    const double dev = fmax(fabs(mx - mu), fabs(mu - mn)) * (1.0 + 1e-6);
    double* o = a.cs + c * 12;
    o[0] = pow2_scale(dev);
    o[1] = pow2_scale(fmax(mx * mx, mn * mn) * (1.0 + 1e-6));
    o[2] = pow2_scale(dev * a.ycen_absmax * (1.0 + 1e-6));
    o[9] = mu;
    if (a.recip) {
        const double mug = (double)(float)(sg / (double)a.n);
        const double gdev = fmax(fabs(gmx - mug), fabs(mug - gmn)) * (1.0 + 1e-6);
        o[3] = pow2_scale(gdev);
        o[4] = pow2_scale(fmax(gmx * gmx, gmn * gmn) * (1.0 + 1e-6));
        o[5] = mug;
    } else {
        o[3] = o[4] = 1.0;
        o[5] = 0.0;
    }
    o[6] = sg;
    o[7] = sgg;
    o[8] = sgy;
}

__global__ void absmax_kernel(const float* __restrict__ v, int64_t n, unsigned* out_bits) {
    float m = 0.0f;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(v[r]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));  // non-negative floats order as uints
}

__device__ __forceinline__ void split16(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));  // v - hi is exact in fp32
}

struct GramPrepArgs {
    const float* x;           // column-major, ld rows per column
    int64_t ld, n, f, fp;     // fp: row length of the planes (f rounded up to 64)
    const float* ycen;
    const double* cs;
    float eps;
    int write_x, write_g;     // which plane groups to write
    __half* planes;           // plane p: [ld][fp] at planes + p * ld * fp
};

struct ColConst {
    float sx, sq, sw, sg, sgq, mug, mu;
    bool valid;
};

__device__ __forceinline__ ColConst col_const(const double* cs, int64_t c, int64_t f) {
    ColConst k{0, 0, 0, 0, 0, 0, 0, c < f};
    if (k.valid) {
        const double* s = cs + c * 12;
        k.sx = (float)s[0]; k.sq = (float)s[1]; k.sw = (float)s[2];
        k.sg = (float)s[3]; k.sgq = (float)s[4]; k.mug = (float)s[5]; k.mu = (float)s[9];
    }
    return k;
}

// Column-major fp32 -> row-major fp16 planes through a 64-column x 32-row shared-memory
// tile; each thread writes two adjacent columns (__half2, 128 B per warp store).  Rows at or
// beyond n and columns at or beyond f are zero in every plane.
__global__ void __launch_bounds__(256) gram_prep_kernel(GramPrepArgs a) {
    __shared__ __align__(8) float xs[32][66];   // [row][column], even pitch for float2 reads
    __shared__ float ys[32];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int64_t n_ct = a.fp / 64, total = n_ct * (a.ld / 32);
    const int64_t plane = a.ld * a.fp;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x) {
        const int64_t c0 = (t % n_ct) * 64, r0 = (t / n_ct) * 32;
        __syncthreads();
        #pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int64_t c = c0 + ty + 8 * k, r = r0 + tx;
            xs[tx][ty + 8 * k] = (c < a.f && r < a.n) ? a.x[c * a.ld + r] : 0.0f;
        }
        if (ty == 0) ys[tx] = a.ycen[r0 + tx];
        __syncthreads();
        const int64_t c = c0 + 2 * tx;
        const ColConst k0 = col_const(a.cs, c, a.f), k1 = col_const(a.cs, c + 1, a.f);
        #pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int rr = ty + 8 * k;
            const int64_t r = r0 + rr;
            const bool rv = r < a.n;
            const float2 xv = *reinterpret_cast<const float2*>(&xs[rr][2 * tx]);
            const float yv = ys[rr];
            const int64_t o = r * a.fp + c;
            const bool v0 = rv && k0.valid, v1 = rv && k1.valid;
            const __half z = __float2half_rn(0.f);
            if (a.write_x) {
                __half h[6][2];
                #pragma unroll
                for (int q = 0; q < 6; ++q) h[q][0] = h[q][1] = z;
                if (v0) {
                    const float ap = xv.x - k0.mu;
                    split16(ap * k0.sx, h[0][0], h[1][0]);
                    split16(xv.x * xv.x * k0.sq, h[2][0], h[3][0]);
                    split16(ap * yv * k0.sw, h[4][0], h[5][0]);
                }
                if (v1) {
                    const float ap = xv.y - k1.mu;
                    split16(ap * k1.sx, h[0][1], h[1][1]);
                    split16(xv.y * xv.y * k1.sq, h[2][1], h[3][1]);
                    split16(ap * yv * k1.sw, h[4][1], h[5][1]);
                }
                const int pl[6] = {P_XH, P_XL, P_QH, P_QL, P_WH, P_WL};
                #pragma unroll
                for (int q = 0; q < 6; ++q)
                    *reinterpret_cast<__half2*>(&a.planes[pl[q] * plane + o]) = __halves2half2(h[q][0], h[q][1]);
            }
            if (a.write_g) {
                __half h[4][2];
                #pragma unroll
                for (int q = 0; q < 4; ++q) h[q][0] = h[q][1] = z;
                if (v0) {
                    const float gv = safe_recip(xv.x, a.eps);
                    split16((gv - k0.mug) * k0.sg, h[0][0], h[1][0]);
                    split16(gv * gv * k0.sgq, h[2][0], h[3][0]);
                }
                if (v1) {
                    const float gv = safe_recip(xv.y, a.eps);
                    split16((gv - k1.mug) * k1.sg, h[0][1], h[1][1]);
                    split16(gv * gv * k1.sgq, h[2][1], h[3][1]);
                }
                const int pl[4] = {P_GH, P_GL, P_GQH, P_GQL};
                #pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<__half2*>(&a.planes[pl[q] * plane + o]) = __halves2half2(h[q][0], h[q][1]);
            }
        }
    }
}

// ---- reduce: chunks -> raw moments in the 64-tile layout of select.cu ----------------

struct GramReduceArgs {
    const float* partial;
    int n_chunks, n_tiles128;
    const int* lut;           // [nb128 * nb128] 128-tile index or -1
    int nb128;
    const TileCoord* tiles64;
    int n_tiles64;
    int64_t f, n;
    const double* colstats;   // raw columns: sum, sumsq, sum*ycen, mean
    const double* cs;         // scales + g statistics
    int recip;
    double* moments;          // [1][n_tiles64][3][4096]
};

// grid (n_tiles64, 16): 256 pairs of one 64-tile per CTA, consecutive threads on
// consecutive rows m of the partials (coalesced), chunks added in a fixed order.
__global__ void __launch_bounds__(256) gram_reduce_kernel(GramReduceArgs a) {
    const int t = blockIdx.x;
    const TileCoord tc = a.tiles64[t];
    const int I = tc.bi >> 1, J = tc.bj >> 1;
    const int t128 = a.lut[I * a.nb128 + J];
    const double n = (double)a.n;
    double* out = a.moments + (int64_t)t * 3 * kTilePairs;
    const int q = blockIdx.y * blockDim.x + threadIdx.x;   // 0 .. 4095
    const int lj = q / kTile, li = q % kTile;
    const int e = li * kTile + lj;
    const int m = (tc.bi & 1) * kTile + li, nn = (tc.bj & 1) * kTile + lj;
    const int64_t i = (int64_t)tc.bi * kTile + li, j = (int64_t)tc.bj * kTile + lj;
    double S1 = 0.0, Q = 0.0, S3 = 0.0;
    if (t128 >= 0 && i < a.f && j < a.f) {
        double C = 0.0, W = 0.0;
        const float* p = a.partial + (int64_t)t128 * 3 * kGT * kGT + (int64_t)nn * kGT + m;
        const int64_t cstride = (int64_t)a.n_tiles128 * 3 * kGT * kGT;
        #pragma unroll 4
        for (int ch = 0; ch < a.n_chunks; ++ch) {
            const float* pc = p + ch * cstride;
            C += (double)pc[0];
            Q += (double)pc[(int64_t)kGT * kGT];
            W += (double)pc[(int64_t)2 * kGT * kGT];
        }
        const double* ci = a.cs + i * 12;
        const double* cj = a.cs + j * 12;
        const double mua = ci[9];                 // the mean the planes subtracted (fp32)
        const double Sa = a.colstats[i * 4 + 0], Ua = a.colstats[i * 4 + 2];
        double mub, Sb, Ub, sB, sQB;
        if (a.recip) {
            mub = cj[5]; Sb = cj[6]; Ub = cj[8]; sB = cj[3]; sQB = cj[4];
        } else {
            mub = cj[9]; Sb = a.colstats[j * 4 + 0]; Ub = a.colstats[j * 4 + 2];
            sB = cj[0]; sQB = cj[1];
        }
        C /= ci[0] * sB;
        Q /= ci[1] * sQB;
        W /= ci[2] * sB;
        // undo the centring: a = a' + mean_a, g(b) = b' + mean_b
        const double sa_c = Sa - n * mua, sb_c = Sb - n * mub;   // sum a', sum b' (~0)
        S1 = C + mua * sb_c + mub * sa_c + n * mua * mub;
        // sum a b ycen = W + mean_a sum b' ycen + mean_b sum a' ycen + mean_a mean_b sum ycen;
        // sum ycen is the rounding residue of fl32(y - mean y) (~1e-8 sqrt(n)) and is dropped,
        // which also makes sum a' ycen = sum a ycen.
        S3 = W + mua * Ub + mub * Ua;
    }
    out[e] = S1;
    out[kTilePairs + e] = Q;
    out[2 * kTilePairs + e] = S3;
}

// ---- host helpers ---------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

bool make_plane_map(CUtensorMap* map, const __half* base, int64_t ld, int64_t fp) {
    auto enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)fp, (cuuint64_t)ld};
    cuuint64_t strides[1] = {(cuuint64_t)fp * sizeof(__half)};
    cuuint32_t box[2] = {64, (cuuint32_t)kGK};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void*)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Rows one CTA accumulates in fp32 before its partial goes to fp64 (8192 by default;
// GAFIME_GRAM_CHUNK_ROWS overrides it for accuracy studies).
int64_t max_chunk_rows() {
    static int64_t v = -1;
    if (v < 0) {
        const char* s = getenv("GAFIME_GRAM_CHUNK_ROWS");
        int64_t x = s ? atoll(s) : kMaxChunkRows;
        v = std::max<int64_t>(kRowPad, (x / kRowPad) * kRowPad);
    }
    return v;
}

}  // namespace

bool gram_path_enabled(const Bucket& b) {
    static int env = -1;
    if (env < 0) {
        const char* v = getenv("GAFIME_PAIR_MOMENTS");
        env = (v && std::string(v) == "cuda-core") ? 0 : 1;
    }
    if (!env) return false;
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, b.device);
    return major == 10 && encode_fn() != nullptr;
}

cudaError_t launch_gram_moments(Bucket& b, const ColumnStats& cs, const TileCoord* d_tiles64,
                                const std::vector<TileCoord>& tiles64, bool recip, float eps,
                                double* d_moments, cudaStream_t stream, int* host_err, int prep_mode) {
    *host_err = 0;
    const int64_t f = b.f, ld = b.ld, n = b.n;
    const int64_t fp = (f + 63) / 64 * 64;
    const int nb128 = (int)((f + kGT - 1) / kGT);
    // 128-tiles that cover this shard's 64-tiles
    std::vector<int> lut((size_t)nb128 * nb128, -1);
    std::vector<TileCoord> t128;
    for (const TileCoord& t : tiles64) {
        int I = t.bi >> 1, J = t.bj >> 1;
        if (lut[(size_t)I * nb128 + J] < 0) {
            lut[(size_t)I * nb128 + J] = (int)t128.size();
            t128.push_back({I, J});
        }
    }
    const int nt = (int)t128.size();
    if (nt == 0) return cudaSuccess;
    // row chunks: <= max_chunk_rows() rows, enough CTAs for every SM
    int64_t want = std::max<int64_t>(1, (4 * (int64_t)b.sm_count + nt - 1) / nt);
    int64_t chunk = (ld + want - 1) / want;
    chunk = std::min<int64_t>(max_chunk_rows(), std::max<int64_t>(1024, chunk));
    chunk = (chunk + kRowPad - 1) / kRowPad * kRowPad;
    const int n_chunks = (int)((ld + chunk - 1) / chunk);

    // scratch: planes | partial | lut | tiles128 | colparts | cs | err/absmax.  The plane
    // region has room for the divide planes whenever this call or the next one needs them,
    // so both moment groups of one scoring call see the same layout.
    const bool g_planes = recip || prep_mode != GRAM_PREP_OWN;
    const int n_planes = g_planes ? P_COUNT : P_GH;
    size_t planes_bytes = (size_t)n_planes * fp * ld * sizeof(__half);
    size_t off_part = (planes_bytes + 255) / 256 * 256;
    size_t part_bytes = (size_t)n_chunks * nt * 3 * kGT * kGT * sizeof(float);
    size_t off_lut = (off_part + part_bytes + 255) / 256 * 256;
    size_t off_t128 = (off_lut + lut.size() * sizeof(int) + 255) / 256 * 256;
    int splits = (int)std::max<int64_t>(1, std::min<int64_t>((4 * (int64_t)b.sm_count + f - 1) / f,
                                                             (n + 4095) / 4096));
    splits = std::min(splits, 256);
    size_t off_colp = (off_t128 + t128.size() * sizeof(TileCoord) + 255) / 256 * 256;
    size_t off_cs = (off_colp + (size_t)f * splits * sizeof(GramColPart) + 255) / 256 * 256;
    size_t off_err = (off_cs + (size_t)f * 12 * sizeof(double) + 255) / 256 * 256;
    size_t total = off_err + 256;
    cudaError_t e = ensure(b.gram, total);
    if (e != cudaSuccess) return e;
    char* base = (char*)b.gram.ptr;
    __half* planes = (__half*)base;
    float* partial = (float*)(base + off_part);
    int* d_lut = (int*)(base + off_lut);
    TileCoord* d_t128 = (TileCoord*)(base + off_t128);
    GramColPart* colp = (GramColPart*)(base + off_colp);
    double* d_cs = (double*)(base + off_cs);
    int* d_err = (int*)(base + off_err);
    unsigned* d_absmax = (unsigned*)(base + off_err + 64);

    e = cudaMemcpyAsync(d_lut, lut.data(), lut.size() * sizeof(int), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_t128, t128.data(), t128.size() * sizeof(TileCoord), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_err, 0, 128, stream);
    if (e != cudaSuccess) return e;

    if (prep_mode != GRAM_PREP_DONE) {
        // operand statistics, scales and planes (both groups' planes when asked)
        const bool both = prep_mode == GRAM_PREP_BOTH;
        int64_t span = ((n + splits - 1) / splits + 255) / 256 * 256;
        {
            KernelTimer timer(stream, GAFIME_KERNEL_GRAM_PREP);
            e = cudaMemsetAsync(d_absmax, 0, sizeof(unsigned), stream);
            if (e != cudaSuccess) return e;
            absmax_kernel<<<2 * b.sm_count, 256, 0, stream>>>(cs.d_ycen, ld, d_absmax);
            gram_colstats_kernel<<<dim3((unsigned)f, (unsigned)splits), 256, 0, stream>>>(
                cs.d_x, ld, n, cs.d_ycen, (recip || both) ? 1 : 0, eps, span, colp);
        }
        unsigned h_absmax = 0;
        e = cudaMemcpyAsync(&h_absmax, d_absmax, sizeof(unsigned), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return e;
        float yabs = 0.0f;
        memcpy(&yabs, &h_absmax, sizeof(float));
        GramScaleArgs sa;
        sa.part = colp;
        sa.splits = splits;
        sa.f = f;
        sa.n = n;
        sa.colstats = cs.d_col;
        sa.ycen_absmax = (double)yabs;
        sa.recip = (recip || both) ? 1 : 0;
        sa.cs = d_cs;
        GramPrepArgs pa;
        pa.x = cs.d_x;
        pa.ld = ld;
        pa.n = n;
        pa.f = f;
        pa.fp = fp;
        pa.ycen = cs.d_ycen;
        pa.cs = d_cs;
        pa.eps = eps;
        pa.write_x = 1;
        pa.write_g = (recip || both) ? 1 : 0;
        pa.planes = planes;
        KernelTimer timer(stream, GAFIME_KERNEL_GRAM_PREP);
        gram_scale_kernel<<<(unsigned)((f + 127) / 128), 128, 0, stream>>>(sa);
        const int64_t prep_tiles = (fp / 64) * (ld / 32);
        const int prep_blocks = (int)std::min<int64_t>(prep_tiles, 32 * (int64_t)b.sm_count);
        gram_prep_kernel<<<prep_blocks, 256, 0, stream>>>(pa);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }

    GramMaps maps;
    for (int p = 0; p < P_COUNT; ++p)
        if (!make_plane_map(&maps.m[p], planes + (size_t)(p < n_planes ? p : 0) * fp * ld, ld, fp))
            return cudaErrorInvalidValue;
    GramArgs ga;
    ga.tiles = d_t128;
    ga.n_tiles = nt;
    ga.chunk_rows = chunk;
    ga.rows = ld;
    const int a_planes[kNumA] = {P_XH, P_XL, P_QH, P_QL, P_WH, P_WL};
    const int b_planes[kNumB] = {recip ? P_GH : P_XH, recip ? P_GL : P_XL, recip ? P_GQH : P_QH,
                                 recip ? P_GQL : P_QL};
    for (int o = 0; o < kNumA; ++o) ga.a_plane[o] = a_planes[o];
    for (int o = 0; o < kNumB; ++o) ga.b_plane[o] = b_planes[o];
    ga.partial = partial;
    ga.err = d_err;
    const size_t smem = (size_t)kGStages * kStageBytes + 1024 + 256;
    e = cudaFuncSetAttribute(gram_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    {
        KernelTimer timer(stream, GAFIME_KERNEL_GRAM_TC);
        gram_tile_kernel<<<dim3((unsigned)nt, (unsigned)n_chunks), kGramThreads, smem, stream>>>(maps, ga);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    GramReduceArgs ra;
    ra.partial = partial;
    ra.n_chunks = n_chunks;
    ra.n_tiles128 = nt;
    ra.lut = d_lut;
    ra.nb128 = nb128;
    ra.tiles64 = d_tiles64;
    ra.n_tiles64 = (int)tiles64.size();
    ra.f = f;
    ra.n = n;
    ra.colstats = cs.d_col;
    ra.cs = d_cs;
    ra.recip = recip ? 1 : 0;
    ra.moments = d_moments;
    {
        KernelTimer timer(stream, GAFIME_KERNEL_GRAM_REDUCE);
        gram_reduce_kernel<<<dim3((unsigned)tiles64.size(), kTilePairs / 256), 256, 0, stream>>>(ra);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    int h_err = 0;
    e = cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    *host_err = h_err;
    return e;
}

}  // namespace gafime
