// gram.cu -- pair moments as tcgen05 Gram tiles (sm_100a tensor cores).
//
// For a 128 x 128 block of column pairs (i in block I, j in block J) the three pair
// moments are dense contractions over rows:
//     C = sum a'b'            (centred columns a' = a - mean_a, b' = g(b) - mean_g)
//     Q = sum a^2 g(b)^2      (raw squares)
//     W = sum (a' ycen) b'    (ycen = y - mean y)
// with g = identity (multiply; add / subtract reuse C) or g(b) = 1/safe(b) (divide).
// They are computed by tcgen05.mma kind::f16 with fp32 accumulators in tensor memory
// (TMEM columns 0-127: C, 128-255: W, 256-383: Q).  Each fp16 operand is a 2-term split of a
// per-column power-of-two-scaled value (|value| <= 2^14, ~22 significant bits):
//     XH/XL = split(s_x a'),  QH/QL = split(s_q a^2)                                  (A)
//     BH/BL = split(s b'),  WBH/WBL = split(s b' * s_y ycen),  BQH/BQL = split(s_q g(b)^2) (B)
// and each Gram is hi.hi + hi.lo + lo.hi (the lo.lo term is below fp32 rounding).  C and W
// share their A operand, so [BH|WBH] and [BL|WBL] are 256-row B operands of N = 256 MMAs:
// six MMAs per 16-row step.  One fp16 term per operand is not enough when a few rows
// dominate a sum (heavy tails, near-zero divisors): their 2^-12 rounding would not average
// out.
//
// One CTA = one tile x one chunk of <= 8192 rows (each fp32 accumulation stays short), 18
// warps:
//   warp 0      TMA: raw fp32 column tiles (128 columns x 16 rows, 64-byte swizzle, no
//               multicast) of the A block and, off the diagonal, the B block, plus 16 scaled
//               ycen values (plain bulk copy) -> 8-stage raw ring
//   warp 1      TMEM allocation; one thread waits for a super-step (two consecutive steps'
//               operands), issues their twelve MMAs (A operands from tensor memory, B
//               operands from shared memory) and commits the pair of operand stages back
//               to its "empty" barrier
//   warps 2-17  two converter groups of 8 warps, taking alternate steps; one column of each
//               block and one 8-row K half per thread, in the TMEM lane quarter of its
//               warp: centre, scale and split the values, write the four A rows to tensor
//               memory (tcgen05.st) and the six B rows to K-major fp16 tiles (32-byte
//               swizzle) in shared memory, 4-stage operand ring handed out in pairs.  The
//               MMA thread shares its SM sub-partition with four converter warps, so its
//               loop is issue-bound: one wait and commit per step (instead of per pair)
//               kept the tensor pipe ~40 % idle.  Diagonal tiles of the
//               multiply group load and convert one block only.  After the last step group 0
//               drains TMEM (tcgen05.ld) into fp32 chunk partials.
// Keeping A in tensor memory halves the shared-memory reads of the MMAs (shared-memory
// bandwidth, not the tensor pipe, bounds a 128 x 128 tile with both operands there).  The
// raw fp32 matrix is read once per tile and chunk (concurrent tiles of one chunk share it
// through L2); no operand planes exist in HBM.
// Wide tables take gram_planes_kernel instead (below): the B operands are converted once per
// call into fp16 planes in HBM and TMA-loaded, and only the A block is converted in-kernel.
// gram_reduce_kernel then adds the chunk partials in fp64 in a fixed order, undoes the scales
// and the centring, and writes the raw moments S1 = sum a g(b), S2 = Q, S3 = sum a g(b) ycen
// that select.cu's epilogue scores.
//
// Every mbarrier wait is bounded: on timeout the thread records an error code in err[0] and
// stops; the MMA warp still commits the accumulator barrier, the producer drains its copies,
// and the CTA frees its TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "engine.h"

namespace gafime {

namespace {

constexpr int kGT = 128;                      // Gram tile edge (columns)
constexpr int kGK = 16;                       // rows per step (one MMA K step)
constexpr int kRawStages = 8;
constexpr int kOpStages = 4;                  // A operands in TMEM + B operands in shared memory
constexpr int kRawBox = kGT * kGK * 4;        // one fp32 column tile: 128 columns x 16 rows
constexpr int kRawStageBytes = 2 * kRawBox;   // A block + B block
constexpr int kYsBytes = 64;                  // 16 scaled ycen values
constexpr int kOpBytes = kGT * kGK * 2;       // one fp16 operand tile: 128 columns x 16 rows
// B stage: [BH | WBH] [BL | WBL] (256-row N = 256 operands) BQH BQL
constexpr int kBH = 0, kBL = 2 * kOpBytes, kBQH = 4 * kOpBytes, kBQL = 5 * kOpBytes;
constexpr int kBStageBytes = 6 * kOpBytes;
constexpr uint32_t kTmemCW = 0;               // [C | W] accumulators (256 columns)
constexpr uint32_t kTmemQ = 256;              // Q accumulator (128 columns)
constexpr uint32_t kTmemA = 384;              // A operand stages after the accumulators
constexpr uint32_t kTmemAStride = 32;         // XH XL QH QL: 8 columns each
constexpr int kConvWarps = 8;                 // warps per converter group (column x K half per thread)
constexpr int kGroups = 2;                    // converter groups, interleaved over the steps
constexpr int kGramThreads = (2 + kGroups * kConvWarps) * 32;
// Super-steps: the operand ring hands out pairs of consecutive steps (step 2j from converter
// group 0, step 2j + 1 from group 1), so the MMA thread waits, and commits, once per twelve
// MMAs.  Its per-step loop competes for issue slots with the converter warps of its SM
// sub-partition; one wait and commit per step cost about 40 % of the tensor pipe's time.
constexpr int kSuper = 2;                     // steps per super-stage
constexpr int kSuperStages = kOpStages / kSuper;
static_assert(kSuper == kGroups && kOpStages % kSuper == 0, "a super-step is one step of each converter group");
constexpr uint32_t kTmemCols = 512;
constexpr long long kSpinLimit = 1LL << 24;
constexpr uint32_t kSuspendNs = 20000;           // try_wait suspend-time hint
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s: a wait this long is a fault
constexpr int64_t kMaxChunkRows = 8192;
constexpr size_t kGramSmem = (size_t)kRawStages * (kRawStageBytes + kYsBytes) + (size_t)kOpStages * kBStageBytes +
                             1024 + 256;
static_assert(kGramSmem <= 232448, "shared memory per CTA");
static_assert(kTmemA + kOpStages * kTmemAStride <= kTmemCols, "tensor memory columns");

struct GramArgs {
    const TileCoord* tiles;   // 128-blocks (bi, bj), bi <= bj
    int n_tiles;
    int64_t chunk_rows;       // multiple of kGK
    int64_t rows;             // padded rows (ld)
    int64_t n, f;             // valid rows and columns
    const float* ys;          // [ld] ycen * s_y (s_y: power of two, |ys| <= 1), zero beyond n
    const double* cs;         // per-column scales and means (12 doubles per column)
    int recip;                // B side is 1/safe(b)
    float eps;
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
    // the suspend-time hint lets the thread sleep until the phase completes (or the hint
    // expires) instead of spinning on the issue slots the converter warps need
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kSuspendNs)
        : "memory");
    return ok != 0;
}

// Non-blocking test: the single producer and MMA threads poll, so they go on as soon as the
// phase completes (a thread suspended in try_wait may be woken later than that)
__device__ __forceinline__ bool mbar_try_spin(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: true when the phase completed, false (error recorded) after kWaitLimitNs of
// wall time or kSpinLimit attempts, whichever comes first.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (long long i = 1; i < kSpinLimit; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitLimitNs) break;
    }
    atomicCAS(err, 0, code);
    return false;
}

// Bounded wait of the single producer / MMA threads: polls without suspending
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, int* err, int code) {
    if (mbar_try_spin(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (long long i = 1; i < kSpinLimit; ++i) {
        if (mbar_try_spin(bar, parity)) return true;
        if ((i & 15) == 0 && global_ns() - t0 > kWaitLimitNs) break;
    }
    atomicCAS(err, 0, code);
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"((uint64_t)map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// Plain bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"((uint64_t)src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile with the 32-byte swizzle: 128 rows (columns of X) of 32 B (16 fp16
// along K), 8-row groups 256 B apart (SBO), LBO unused (1), descriptor version 1, layout 6.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)6 << 61);
}

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, N = 128, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kGT >> 3) << 17) |
                            ((uint32_t)(kGT >> 4) << 24);
// the same with N = 256: B = [b' rows | (s_y ycen) b' rows], D = [C | W]
constexpr uint32_t kIdesc256 = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(2 * kGT >> 3) << 17) |
                               ((uint32_t)(kGT >> 4) << 24);

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void fence_async_smem() {
    // make generic-proxy shared-memory writes visible to the tensor cores (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1 / safe(v) with the hardware reciprocal (max error 1 ulp; the operand split keeps 22
// bits of it).  The statistics pass and the operand converters both use this function, so
// the centring means are those of the values the tensor cores multiply.  Subnormals flush
// to zero: a result for |v| >= 2^126, an input only when eps < 2^-126.
__device__ __forceinline__ float safe_recip(float v, float eps) {
    float d = fabsf(v) < eps ? copysignf(eps, v) : v;
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
    return r;
}

// A operand in tensor memory (lane = row m, 8 columns = 16 fp16 along K), B in shared memory
__device__ __forceinline__ void umma_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate)
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

// ---- the fused Gram kernel ---------------------------------------------------------

// Bounded wait by lane 0 of a warp; the shuffle makes the outcome warp-uniform and orders
// the other lanes' later accesses after lane 0's acquire.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int* err, int code, int lane) {
    int ok = 1;
    if (lane == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok != 0;
}

// The same with lane 0 polling (test_wait) instead of suspending: the fused kernel's
// converters sit on the chain MMA completion -> operand stores -> next MMAs, where a
// suspended thread's wake-up latency costs tensor-pipe time.
__device__ __forceinline__ bool warp_wait_poll(uint32_t bar, uint32_t parity, int* err, int code, int lane) {
    int ok = 1;
    if (lane == 0) ok = mbar_wait_spin(bar, parity, err, code) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok != 0;
}

// 8 consecutive rows (one K half) of one column as hi and lo fp16 pairs
struct Split8 {
    uint32_t hi[4], lo[4];
};

// Packed fp32 pairs (two rows of one column) for the sm_100 f32x2 instructions; each lane
// is rounded exactly like the scalar operation.
__device__ __forceinline__ uint64_t pk(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 upk(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// 2-term split of 8 values (4 packed pairs): hi = fp16(v), lo = fp16(v - hi) (v - hi is
// exact in fp32, and |v - hi| <= 2^-11 |v|, so hi + lo carries ~22 significant bits).
__device__ __forceinline__ void split8(const uint64_t (&v)[4], Split8& s) {
    #pragma unroll
    for (int p = 0; p < 4; ++p) {
        const float2 f = upk(v[p]);
        __half2 h = __floats2half2_rn(f.x, f.y);
        const float2 hf = __half22float2(h);
        const float2 d = upk(sub2(v[p], pk(hf.x, hf.y)));
        __half2 l = __floats2half2_rn(d.x, d.y);
        s.hi[p] = *reinterpret_cast<uint32_t*>(&h);
        s.lo[p] = *reinterpret_cast<uint32_t*>(&l);
    }
}

// Rows 8h .. 8h+7 of column m of a raw fp32 tile (64-byte swizzle: the 16-byte chunk q of
// column m sits at position q ^ ((m >> 1) & 3)).
__device__ __forceinline__ void load_raw8(const unsigned char* tile, int m, int h, float (&x)[8]) {
    const int sw = (m >> 1) & 3;
    #pragma unroll
    for (int q = 0; q < 2; ++q) {
        float4 u = *reinterpret_cast<const float4*>(tile + m * 64 + 16 * ((2 * h + q) ^ sw));
        x[4 * q] = u.x;
        x[4 * q + 1] = u.y;
        x[4 * q + 2] = u.z;
        x[4 * q + 3] = u.w;
    }
}

// K half h of row m of a K-major fp16 tile with the 32-byte swizzle (halves swapped when
// bit 2 of m is set)
__device__ __forceinline__ void store_half(unsigned char* tile, int m, int h, const uint32_t (&v)[4]) {
    *reinterpret_cast<uint4*>(tile + m * 32 + 16 * (h ^ ((m >> 2) & 1))) = make_uint4(v[0], v[1], v[2], v[3]);
}

// 4 consecutive 32-bit TMEM columns of this thread's lane (one K half of an A row)
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3])
                 : "memory");
}

// Per-column constants of one converter thread (all zero for columns beyond f).
struct ConvCols {
    float mus_a, sx_a, sq_a;   // A block: mean * s_x, s_x, s_q
    float mus_b, sx_b, sq_b;   // B block: mean * s, s, s_q of b (multiply) or g(b) (divide)
};

// Operand rows of one column and K half for one step
struct StepOps {
    Split8 x, q;        // A: s_x a',  s_q a^2
    Split8 b, wb, bq;   // B: s b',    (s b') (s_y ycen),  s_q g(b)^2
};

// Convert K half h of column m for one step (A block, and the B block when kB).  kMask
// zeroes rows at or beyond `valid`.  fma(x, s, -mean*s) equals fl(x - mean) * s exactly (s
// is a power of two).  Rows are processed in packed pairs (f32x2).
template <bool kMask, bool kB, bool kRecip>
__device__ __forceinline__ void convert_step(const unsigned char* raw, const unsigned char* ysm, int m, int h,
                                             int valid, const ConvCols& k, float eps, StepOps& o,
                                             int b_off = kRawBox) {
    float x[8];
    uint64_t x2[4], v2[4], t2[4];
    load_raw8(raw, m, h, x);
    #pragma unroll
    for (int p = 0; p < 4; ++p) x2[p] = pk(x[2 * p], x[2 * p + 1]);
    const uint64_t sx = pk(k.sx_a, k.sx_a), nmu = pk(-k.mus_a, -k.mus_a), sq = pk(k.sq_a, k.sq_a);
    #pragma unroll
    for (int p = 0; p < 4; ++p) {
        v2[p] = fma2(x2[p], sx, nmu);              // C: s_x (a - mean)
        t2[p] = mul2(mul2(x2[p], x2[p]), sq);      // Q: s_q a^2
        if (kMask) {
            const bool v0 = 8 * h + 2 * p < valid, v1 = 8 * h + 2 * p + 1 < valid;
            const float2 c = upk(v2[p]), q = upk(t2[p]);
            v2[p] = pk(v0 ? c.x : 0.f, v1 ? c.y : 0.f);
            t2[p] = pk(v0 ? q.x : 0.f, v1 ? q.y : 0.f);
        }
    }
    split8(v2, o.x);
    split8(t2, o.q);
    if (kB) {
        load_raw8(raw + b_off, m, h, x);
        if (kRecip) {
            #pragma unroll
            for (int r = 0; r < 8; ++r) x[r] = safe_recip(x[r], eps);
        }
        #pragma unroll
        for (int p = 0; p < 4; ++p) x2[p] = pk(x[2 * p], x[2 * p + 1]);
        const uint64_t sxb = pk(k.sx_b, k.sx_b), nmub = pk(-k.mus_b, -k.mus_b), sqb = pk(k.sq_b, k.sq_b);
        #pragma unroll
        for (int p = 0; p < 4; ++p) {
            v2[p] = fma2(x2[p], sxb, nmub);
            t2[p] = mul2(mul2(x2[p], x2[p]), sqb);
            if (kMask) {
                const bool v0 = 8 * h + 2 * p < valid, v1 = 8 * h + 2 * p + 1 < valid;
                const float2 c = upk(v2[p]), q = upk(t2[p]);
                v2[p] = pk(v0 ? c.x : 0.f, v1 ? c.y : 0.f);
                t2[p] = pk(v0 ? q.x : 0.f, v1 ? q.y : 0.f);
            }
        }
        split8(v2, o.b);
        split8(t2, o.bq);
    }
    {
        // W's B operand: the B block's C operand times s_y ycen (the A block's on the
        // multiply group's diagonal, where B = A)
        const float4 y0 = *reinterpret_cast<const float4*>(ysm + 32 * h);
        const float4 y1 = *reinterpret_cast<const float4*>(ysm + 32 * h + 16);
        v2[0] = mul2(v2[0], pk(y0.x, y0.y));
        v2[1] = mul2(v2[1], pk(y0.z, y0.w));
        v2[2] = mul2(v2[2], pk(y1.x, y1.y));
        v2[3] = mul2(v2[3], pk(y1.z, y1.w));
    }
    split8(v2, o.wb);
}

// Shared-memory and tensor-memory addresses of one converter thread
struct ConvCtx {
    const unsigned char* raw0;   // raw ring
    const unsigned char* ys0;    // scaled ycen ring
    unsigned char* bop0;         // B operand ring
    uint32_t rfull0, rempty0, ofull0, oempty0;
    uint32_t tmem_a;             // tmem + lane quarter + kTmemA + 4h
    int m, h, lane;
    int nk, n_full;              // steps in the chunk; steps with all 16 rows below n
    int64_t rows_left;           // n - first row of the chunk
    float eps;
    int* err;
    int b_off;                   // B raw tile in a stage: kRawBox, or 0 when it is the A tile
};

// The steps k = grp, grp + kGroups, ... of one converter thread.  kB: convert the B block
// (off the multiply group's diagonal); kRecip: the B operand is 1/safe(b).  Step k belongs to
// super-step k / kSuper, whose stage pair ss = (k / kSuper) % kSuperStages holds operand
// stages 2 ss and 2 ss + 1 (= k % kOpStages).  Every warp of both groups waits on every
// phase of each super-stage's "empty" barrier, in order, so its parity waits are sound.
template <bool kB, bool kRecip>
__device__ __forceinline__ void conv_loop(const ConvCtx& c, const ConvCols& kc, int grp) {
    for (int k = grp; k < c.nk; k += kGroups) {
        const int rs = k % kRawStages, os = k % kOpStages;
        const int j = k / kSuper, ss = j % kSuperStages;
        if (!warp_wait_poll(c.rfull0 + 8 * rs, (k / kRawStages) & 1, c.err, 5, c.lane)) return;
        const unsigned char* raw = c.raw0 + rs * kRawStageBytes;
        const unsigned char* ysm = c.ys0 + rs * kYsBytes;
        StepOps o;
        if (k < c.n_full) {
            convert_step<false, kB, kRecip>(raw, ysm, c.m, c.h, kGK, kc, c.eps, o, c.b_off);
        } else {
            const int64_t left = c.rows_left - (int64_t)k * kGK;
            const int valid = left <= 0 ? 0 : (int)left;   // < kGK here
            convert_step<true, kB, kRecip>(raw, ysm, c.m, c.h, valid, kc, c.eps, o, c.b_off);
        }
        {
            // Every value read from the raw stage is now in registers: hand the stage back to
            // the producer before waiting for an operand stage, so the raw ring keeps
            // prefetching while the MMAs drain.  `dep` is computed from every converted word
            // (each depends on the loads of its rows), so no lane reaches the warp barrier,
            // and lane 0 no release, before that lane's shared-memory loads have returned.
            uint32_t dep = 0;
            #pragma unroll
            for (int p = 0; p < 4; ++p) {
                dep ^= o.x.hi[p] ^ o.q.hi[p] ^ o.wb.hi[p];
                if (kB) dep ^= o.b.hi[p] ^ o.bq.hi[p];
            }
            asm volatile("" ::"r"(dep) : "memory");
            __syncwarp();
            if (c.lane == 0) mbar_arrive(c.rempty0 + 8 * rs);
        }
        // the super-stage must be free: the MMAs of super-step j - kSuperStages have completed
        if (j >= kSuperStages && !warp_wait_poll(c.oempty0 + 8 * ss, ((j / kSuperStages) - 1) & 1, c.err, 6, c.lane))
            return;
        tc_fence_after();
        const uint32_t ta = c.tmem_a + (uint32_t)(os * kTmemAStride);
        tmem_st4(ta + 0 * 8, o.x.hi);
        tmem_st4(ta + 1 * 8, o.x.lo);
        tmem_st4(ta + 2 * 8, o.q.hi);
        tmem_st4(ta + 3 * 8, o.q.lo);
        unsigned char* sb = c.bop0 + os * kBStageBytes;
        const Split8& b0 = kB ? o.b : o.x;
        const Split8& b1 = kB ? o.bq : o.q;
        store_half(sb + kBH, c.m, c.h, b0.hi);
        store_half(sb + kBL, c.m, c.h, b0.lo);
        store_half(sb + kBH + kOpBytes, c.m, c.h, o.wb.hi);
        store_half(sb + kBL + kOpBytes, c.m, c.h, o.wb.lo);
        store_half(sb + kBQH, c.m, c.h, b1.hi);
        store_half(sb + kBQL, c.m, c.h, b1.lo);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (c.lane == 0) mbar_arrive(c.ofull0 + 8 * ss);
    }
    if (grp == kGroups - 1 && (c.nk % kSuper) != 0) {
        // the last super-step has no step for this group: arrive for it all the same (after
        // the same wait, so the arrival counts toward that super-step's phase)
        const int j = c.nk / kSuper, ss = j % kSuperStages;
        if (j >= kSuperStages && !warp_wait_poll(c.oempty0 + 8 * ss, ((j / kSuperStages) - 1) & 1, c.err, 6, c.lane))
            return;
        __syncwarp();
        if (c.lane == 0) mbar_arrive(c.ofull0 + 8 * ss);
    }
}

__global__ void __launch_bounds__(kGramThreads, 1)
gram_fused_kernel(const __grid_constant__ CUtensorMap xmap, const GramArgs a) {
    extern __shared__ __align__(1024) unsigned char gsmem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)gsmem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char* raw0 = smem;                                    // raw ring
    unsigned char* bop0 = raw0 + kRawStages * kRawStageBytes;      // B operand ring
    unsigned char* ys0 = bop0 + kOpStages * kBStageBytes;          // scaled ycen ring
    uint64_t* bars = (uint64_t*)(ys0 + kRawStages * kYsBytes);
    // raw_full[R], raw_empty[R], op_full[O], op_empty[O], accum
    const uint32_t rfull0 = smem_u32(bars), rempty0 = smem_u32(bars + kRawStages);
    const uint32_t ofull0 = smem_u32(bars + 2 * kRawStages), oempty0 = smem_u32(bars + 2 * kRawStages + kOpStages);
    const uint32_t accum = smem_u32(bars + 2 * kRawStages + 2 * kOpStages);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kRawStages + 2 * kOpStages + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileCoord tc = a.tiles[blockIdx.x];
    // diagonal tiles load one raw block (A and B columns are the same); the multiply group's
    // also converts it once (its B operand is A's)
    const bool raw_same = tc.bi == tc.bj;
    const bool b_same = raw_same && !a.recip;
    const int64_t r0 = (int64_t)blockIdx.y * a.chunk_rows;
    const int64_t r1 = min(r0 + a.chunk_rows, a.rows);
    const int nk = r1 > r0 ? (int)((r1 - r0) / kGK) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRawStages; ++s) {
            mbar_init(rfull0 + 8 * s, 1);
            mbar_init(rempty0 + 8 * s, kConvWarps);
        }
        for (int s = 0; s < kSuperStages; ++s) {
            mbar_init(ofull0 + 8 * s, kConvWarps * kGroups);   // one arrival per converter warp
            mbar_init(oempty0 + 8 * s, 1);
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
            // producer: raw fp32 column tiles + 16 scaled ycen values per step
            const uint32_t bytes = (raw_same ? (uint32_t)kRawBox : (uint32_t)kRawStageBytes) + (uint32_t)(kGK * 4);
            int issued = 0;
            bool ok = true;
            for (int k = 0; k < nk; ++k) {
                const int s = k % kRawStages;
                if (k >= kRawStages && !(ok = mbar_wait_spin(rempty0 + 8 * s, ((k / kRawStages) - 1) & 1, a.err, 1)))
                    break;
                const uint32_t full = rfull0 + 8 * s;
                mbar_expect_tx(full, bytes);
                const uint32_t st = smem_u32(raw0 + s * kRawStageBytes);
                const int64_t row = r0 + (int64_t)k * kGK;
                tma_load_2d(st, &xmap, full, (int)row, tc.bi * kGT);
                if (!raw_same) tma_load_2d(st + kRawBox, &xmap, full, (int)row, tc.bj * kGT);
                bulk_load(smem_u32(ys0 + s * kYsBytes), a.ys + row, (uint32_t)(kGK * 4), full);
                ++issued;
            }
            if (!ok)
                for (int k = max(0, issued - kRawStages); k < issued; ++k)
                    mbar_wait(rfull0 + 8 * (k % kRawStages), (k / kRawStages) & 1, a.err, 4);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: A operands from tensor memory, B operands from shared memory.  The
            // descriptors of stage s differ from stage 0's only in the start-address field
            // (shared addresses stay below 2^18, so the 14-bit field never carries).
            const uint64_t d0 = umma_desc(smem_u32(bop0));
            const int nj = (nk + kSuper - 1) / kSuper;
            for (int j = 0; j < nj; ++j) {
                // one wait and one commit per super-step (both steps' operands)
                const int ss = j % kSuperStages;
                if (!mbar_wait_spin(ofull0 + 8 * ss, (j / kSuperStages) & 1, a.err, 2)) break;
                tc_fence_after();
                #pragma unroll
                for (int e = 0; e < kSuper; ++e) {
                    const int k = j * kSuper + e;
                    if (k >= nk) break;
                    const int s = ss * kSuper + e;   // == k % kOpStages
                    const uint32_t ta = tmem + kTmemA + (uint32_t)(s * kTmemAStride);
                    const uint64_t ds = d0 + (uint64_t)((s * kBStageBytes) >> 4);
                    // [b' | ycen b'] tiles are 256 consecutive K-major rows: one N = 256 MMA
                    const uint64_t bH = ds + (kBH >> 4), bL = ds + (kBL >> 4);
                    const uint64_t bQH = ds + (kBQH >> 4), bQL = ds + (kBQL >> 4);
                    const uint32_t acc = k > 0 ? 1u : 0u;
                    umma_ta(tmem + kTmemCW, ta + 0 * 8, bH, kIdesc256, acc);   // [C|W]: XH.[BH|WBH]
                    umma_ta(tmem + kTmemCW, ta + 0 * 8, bL, kIdesc256, 1u);    //        XH.[BL|WBL]
                    umma_ta(tmem + kTmemCW, ta + 1 * 8, bH, kIdesc256, 1u);    //        XL.[BH|WBH]
                    umma_ta(tmem + kTmemQ, ta + 2 * 8, bQH, kIdesc, acc);      // Q:     QH.BQH
                    umma_ta(tmem + kTmemQ, ta + 2 * 8, bQL, kIdesc, 1u);       //        QH.BQL
                    umma_ta(tmem + kTmemQ, ta + 3 * 8, bQH, kIdesc, 1u);       //        QL.BQH
                }
                umma_commit(oempty0 + 8 * ss);  // super-stage free once these MMAs have read it
            }
            umma_commit(accum);  // all issued MMAs complete (also on the error path)
        }
    } else {
        // converter groups: group g (warps 2+8g .. 9+8g) converts the steps k = g mod kGroups.
        // Thread = column m of the 128-column blocks (m in the TMEM lane quarter of its warp)
        // and K half h (rows 8h .. 8h+7 of the step).
        const int cw = (warp - 2) % kConvWarps;
        const int grp = (warp - 2) / kConvWarps;
        const int quarter = warp & 3;
        const int h = cw >> 2;
        const int m = quarter * 32 + lane;
        const uint32_t tlane = (uint32_t)(quarter * 32) << 16;
        const int64_t col_a = (int64_t)tc.bi * kGT + m, col_b = (int64_t)tc.bj * kGT + m;
        ConvCols kc{0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (col_a < a.f) {
            const double* c = a.cs + col_a * 12;
            kc.sx_a = (float)c[0];
            kc.sq_a = (float)c[1];
            kc.mus_a = (float)c[9] * kc.sx_a;
        }
        if (col_b < a.f) {
            const double* c = a.cs + col_b * 12;
            const int o = a.recip ? 3 : 0;
            kc.sx_b = (float)c[o];
            kc.sq_b = (float)c[o + 1];
            kc.mus_b = (float)c[a.recip ? 5 : 9] * kc.sx_b;
        }
        ConvCtx cx;
        cx.raw0 = raw0;
        cx.ys0 = ys0;
        cx.bop0 = bop0;
        cx.rfull0 = rfull0;
        cx.rempty0 = rempty0;
        cx.ofull0 = ofull0;
        cx.oempty0 = oempty0;
        cx.tmem_a = tmem + tlane + kTmemA + 4 * h;
        cx.m = m;
        cx.h = h;
        cx.lane = lane;
        cx.nk = nk;
        cx.rows_left = a.n - r0;
        {
            const int64_t full = cx.rows_left / kGK;   // steps whose 16 rows are all below n
            cx.n_full = full <= 0 ? 0 : (full >= nk ? nk : (int)full);
        }
        cx.eps = a.eps;
        cx.err = a.err;
        cx.b_off = raw_same ? 0 : kRawBox;
        if (b_same) conv_loop<false, false>(cx, kc, grp);
        else if (a.recip) conv_loop<true, true>(cx, kc, grp);
        else conv_loop<true, false>(cx, kc, grp);
        if (grp == 0) {
            // group 0 drains the accumulators: TMEM lanes 32*(warp%4) .. +31 are rows m; the
            // two warps of a lane quarter take alternate 32-column chunks
            const bool done = warp_wait(accum, 0, a.err, 3, lane);
            tc_fence_after();
            if (done && nk > 0) {
                float* out = a.partial + ((int64_t)blockIdx.y * a.n_tiles + blockIdx.x) * 3 * kGT * kGT;
                #pragma unroll 1
                for (int idx = h; idx < 3 * kGT / 32; idx += 2) {
                    // partial gram gi = idx / 4 (C, Q, W); its TMEM columns: C at kTmemCW,
                    // W at kTmemCW + 128, Q at kTmemQ
                    const int gi = idx >> 2, cc = (idx & 3) * 32;
                    const uint32_t tcol = (gi == 0 ? kTmemCW : gi == 1 ? kTmemQ : kTmemCW + kGT) + (uint32_t)cc;
                    const int c0 = idx * 32;   // column of the partial's [C | Q | W] layout
                    float tt[32];
                    tmem_ld32(tmem + tlane + tcol, tt);
                    float* op = out + (int64_t)c0 * kGT + m;
                    #pragma unroll
                    for (int c = 0; c < 32; ++c) op[(int64_t)c * kGT] = tt[c];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        // no MMA may still be writing TMEM when it is freed (bounded; returns at once when
        // the accumulator barrier has completed)
        if (lane == 0) mbar_wait(accum, 0, a.err, 7);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

// ---- the wide-table Gram kernel: B operands from per-call planes --------------------------
//
// In a wide table every 128-column block is the B block of many tiles (16 at 2048
// columns), and converting it inside each of them is what binds gram_fused_kernel (the
// converter warps' issue and shared-memory traffic).  Here the B side is converted once per
// call by gram_bplanes_kernel into six fp16 planes in HBM,
//     BH/BL = split(s b'),  WBH/WBL = split((s b') (s_y ycen)),  BQH/BQL = split(s_q g(b)^2)
// (exactly the fused kernel's B-side arithmetic), laid out step-major -- plane, 16-row step,
// column, 16 rows -- with the 32-byte swizzle already applied, so the 128 x 16 operand tile of
// a block and step is one contiguous 4 KB run that a plain bulk copy moves into the K-major
// layout the MMAs read (column-major planes made every tile 128 separate 32-byte pieces 4 MB
// apart, and those loads bound the kernel).  BH and WBH land side by side, so [C | W] is one
// N = 256 MMA as in the fused kernel: three N = 256 and three N = 128 MMAs per 16-row step,
// the same accumulators (TMEM columns 0-127 C, 128-255 W, 256-383 Q) and the same chunk
// partials, reduced by gram_reduce_kernel.  The converters handle the A block only and write
// four A operands (XH/XL = split(s_x a'), QH/QL = split(s_q a^2)) to tensor memory, which
// leaves room for four A stages (the whole of tensor memory): four converter groups work on
// four steps at once.  Two groups of eight warps, each converting every other step, kept the
// tensor pipe ~55 % busy: a group's conversion latency, not bandwidth, paced the steps.
//
// One CTA = one tile x one chunk of <= 8192 rows, 18 warps:
//   warp 0      TMA: raw fp32 A tiles (64-byte swizzle) -> 8-stage ring read by the converters;
//               six fp16 B plane tiles (bulk copies of swizzled 4 KB runs) -> 5-stage ring read
//               by the MMAs
//   warp 1      TMEM allocation; one thread issues the six MMAs of a step, then commits the
//               ring stage (B planes read) and the A stage (TMEM operands read)
//   warps 2-17  four converter groups of 4 warps (one per TMEM lane quarter; a thread
//               converts one A column over the step's 16 rows), group g taking the steps
//               k = g mod 4 into A stage k % 4, so four steps convert at once; groups 0 and
//               1 drain the accumulators at the end
// Every wait is bounded as in gram_fused_kernel.

constexpr int kBPlanes = 6;                                       // BH WBH BL WBL BQH BQL
constexpr int kPRawStages = 8;                                    // raw A tiles (read by the converters)
constexpr int kPBStages = 5;                                      // B plane tiles (read by the MMAs)
constexpr int kPBStageBytes = kBPlanes * kOpBytes;                // 24 KB
constexpr uint32_t kPTmemA = 384;                                 // after C | W | Q
constexpr uint32_t kPTmemAStride = 32;                            // XH XL QH QL: 8 columns each
constexpr int kPAStages = 4;
constexpr int kPGroups = 4;                                       // converter groups (one step each in flight)
constexpr int kPConvWarps = 4;                                    // warps per group: one per TMEM lane quarter
static_assert(2 + kPGroups * kPConvWarps == kGramThreads / 32, "warp roles");
static_assert(kPGroups <= kPAStages, "every group in flight has its own A stage");
// A parity wait is only sound when its barrier's previous phase has completed.  A group's wait
// on raw stage k % kPRawStages follows its own wait on the same stage's previous phase (step
// k - kPRawStages) only when that step was the same group's: the ring depth must be a multiple
// of the number of groups.  (The B ring has one waiter, the MMA thread, in step order.)
static_assert(kPRawStages % kPGroups == 0, "raw ring phases stay with one converter group");
// + up to 1023 bytes to align the base to 1024, + the barriers and the TMEM address slot
constexpr size_t kPBarBytes = (size_t)(2 * kPRawStages + 2 * kPBStages + 2 * kPAStages + 1) * 8 + 8;
constexpr size_t kPlanesSmem = (size_t)kPRawStages * kRawBox + (size_t)kPBStages * kPBStageBytes + 1024 + kPBarBytes;
static_assert(kPlanesSmem <= 232448, "shared memory per CTA");
static_assert(kPTmemA + kPAStages * kPTmemAStride <= kTmemCols, "tensor memory columns");
static_assert(kRawBox % 1024 == 0 && kPBStageBytes % 1024 == 0, "ring stages keep the swizzle alignment");

struct PlanesArgs {
    const TileCoord* tiles;   // 128-blocks (bi, bj), bi <= bj
    int n_tiles;
    int64_t chunk_rows;       // multiple of kGK
    int64_t rows;             // padded rows (ld)
    int64_t n, f;
    int64_t nb;               // 128-column blocks (f_pad / 128)
    const __half* planes;     // [step][block][plane][128][16] fp16, 32-byte swizzled (gram_bplanes_kernel)
    const double* cs;         // per-column scales and means (12 doubles per column)
    float* partial;           // [chunk][tile][3][128 n][128 m]
    int* err;
};

// A operands of one column and K half for one step (rows at or beyond `valid` zeroed).
template <bool kMask>
__device__ __forceinline__ void convert_a(const unsigned char* raw, int m, int h, int valid, float sxa, float nmua,
                                          float sqa, Split8& xo, Split8& qo) {
    float x[8];
    uint64_t x2[4], v2[4], t2[4];
    load_raw8(raw, m, h, x);
    #pragma unroll
    for (int p = 0; p < 4; ++p) x2[p] = pk(x[2 * p], x[2 * p + 1]);
    const uint64_t sx = pk(sxa, sxa), nmu = pk(nmua, nmua), sq = pk(sqa, sqa);
    #pragma unroll
    for (int p = 0; p < 4; ++p) {
        v2[p] = fma2(x2[p], sx, nmu);              // s_x (a - mean)
        t2[p] = mul2(mul2(x2[p], x2[p]), sq);      // s_q a^2
        if (kMask) {
            const bool v0 = 8 * h + 2 * p < valid, v1 = 8 * h + 2 * p + 1 < valid;
            const float2 c = upk(v2[p]), q = upk(t2[p]);
            v2[p] = pk(v0 ? c.x : 0.f, v1 ? c.y : 0.f);
            t2[p] = pk(v0 ? q.x : 0.f, v1 ? q.y : 0.f);
        }
    }
    split8(v2, xo);
    split8(t2, qo);
}

__global__ void __launch_bounds__(kGramThreads, 1)
gram_planes_kernel(const __grid_constant__ CUtensorMap xmap, const PlanesArgs a) {
    extern __shared__ __align__(1024) unsigned char gsmem_raw[];
    unsigned char* smem = (unsigned char*)(((uintptr_t)gsmem_raw + 1023) & ~(uintptr_t)1023);
    unsigned char* rawring = smem;                                // [stage][raw A tile]
    unsigned char* bring = rawring + kPRawStages * kRawBox;       // [stage][BH WBH BL WBL BQH BQL]
    uint64_t* bars = (uint64_t*)(bring + kPBStages * kPBStageBytes);
    // rfull[R], rempty[R], bfull[B], bempty[B], afull[A], aempty[A], accum
    const uint32_t rfull0 = smem_u32(bars), rempty0 = smem_u32(bars + kPRawStages);
    const uint32_t bfull0 = smem_u32(bars + 2 * kPRawStages), bempty0 = smem_u32(bars + 2 * kPRawStages + kPBStages);
    const uint32_t afull0 = smem_u32(bars + 2 * kPRawStages + 2 * kPBStages);
    const uint32_t aempty0 = afull0 + 8 * kPAStages;
    const uint32_t accum = aempty0 + 8 * kPAStages;
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * kPRawStages + 2 * kPBStages + 2 * kPAStages + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const TileCoord tc = a.tiles[blockIdx.x];
    const int64_t r0 = (int64_t)blockIdx.y * a.chunk_rows;
    const int64_t r1 = min(r0 + a.chunk_rows, a.rows);
    const int nk = r1 > r0 ? (int)((r1 - r0) / kGK) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPRawStages; ++s) {
            mbar_init(rfull0 + 8 * s, 1);
            mbar_init(rempty0 + 8 * s, kPConvWarps);   // the step's converter warps
        }
        for (int s = 0; s < kPBStages; ++s) {
            mbar_init(bfull0 + 8 * s, 1);
            mbar_init(bempty0 + 8 * s, 1);             // the step's MMA commit
        }
        for (int s = 0; s < kPAStages; ++s) {
            mbar_init(afull0 + 8 * s, kPConvWarps);
            mbar_init(aempty0 + 8 * s, 1);
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
            int issued = 0;
            bool ok = true;
            for (int k = 0; k < nk; ++k) {
                const int rs = k % kPRawStages, bs = k % kPBStages;
                if (k >= kPRawStages &&
                    !(ok = mbar_wait_spin(rempty0 + 8 * rs, ((k / kPRawStages) - 1) & 1, a.err, 1)))
                    break;
                if (k >= kPBStages && !(ok = mbar_wait_spin(bempty0 + 8 * bs, ((k / kPBStages) - 1) & 1, a.err, 1)))
                    break;
                const int64_t row = r0 + (int64_t)k * kGK;
                mbar_expect_tx(rfull0 + 8 * rs, (uint32_t)kRawBox);
                tma_load_2d(smem_u32(rawring + rs * kRawBox), &xmap, rfull0 + 8 * rs, (int)row, tc.bi * kGT);
                // the six plane tiles of (step, B block): one contiguous 24 KB run, already
                // swizzled -- one copy per step (the copy engine takes few operations at a time,
                // so six 4 KB copies per step starved the pipeline)
                const int64_t step = row / kGK;
                const uint32_t bst = smem_u32(bring + bs * kPBStageBytes);
                mbar_expect_tx(bfull0 + 8 * bs, (uint32_t)kPBStageBytes);
                bulk_load(bst, a.planes + (step * a.nb + tc.bj) * (int64_t)(kPBStageBytes / 2), (uint32_t)kPBStageBytes,
                          bfull0 + 8 * bs);
                ++issued;
            }
            if (!ok) {
                // drain this CTA's copies still in flight before it exits
                for (int k = max(0, issued - kPRawStages); k < issued; ++k)
                    mbar_wait(rfull0 + 8 * (k % kPRawStages), (k / kPRawStages) & 1, a.err, 4);
                for (int k = max(0, issued - kPBStages); k < issued; ++k)
                    mbar_wait(bfull0 + 8 * (k % kPBStages), (k / kPBStages) & 1, a.err, 4);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int k = 0; k < nk; ++k) {
                const int bs = k % kPBStages, as = k % kPAStages;
                if (!mbar_wait_spin(afull0 + 8 * as, (k / kPAStages) & 1, a.err, 2)) break;
                if (!mbar_wait_spin(bfull0 + 8 * bs, (k / kPBStages) & 1, a.err, 2)) break;
                tc_fence_after();
                const uint32_t ta = tmem + kPTmemA + (uint32_t)(as * kPTmemAStride);
                const uint32_t bst = smem_u32(bring + bs * kPBStageBytes);
                // [BH | WBH] and [BL | WBL] are 256 consecutive K-major rows: N = 256 operands
                const uint64_t bH = umma_desc(bst), bL = umma_desc(bst + 2 * kOpBytes);
                const uint64_t bQH = umma_desc(bst + 4 * kOpBytes), bQL = umma_desc(bst + 5 * kOpBytes);
                const uint32_t acc = k > 0 ? 1u : 0u;
                umma_ta(tmem + kTmemCW, ta + 0, bH, kIdesc256, acc);   // [C|W]: XH.[BH|WBH]
                umma_ta(tmem + kTmemCW, ta + 0, bL, kIdesc256, 1u);    //        XH.[BL|WBL]
                umma_ta(tmem + kTmemCW, ta + 8, bH, kIdesc256, 1u);    //        XL.[BH|WBH]
                umma_ta(tmem + kTmemQ, ta + 16, bQH, kIdesc, acc);     // Q:     QH.BQH
                umma_ta(tmem + kTmemQ, ta + 16, bQL, kIdesc, 1u);      //        QH.BQL
                umma_ta(tmem + kTmemQ, ta + 24, bQH, kIdesc, 1u);      //        QL.BQH
                umma_commit(bempty0 + 8 * bs);   // the B planes of this stage have been read
                umma_commit(aempty0 + 8 * as);   // and the A operands of this TMEM stage
            }
            umma_commit(accum);  // all issued MMAs complete (also on the error path)
        }
    } else {
        // converter group grp (warps 2 + 4 grp .. 5 + 4 grp) converts the steps k = grp mod 4,
        // into A stage k % 4; thread = column m of the A block (its TMEM lane), all 16 rows
        const int grp = (warp - 2) / kPConvWarps;
        const int quarter = warp & 3;
        const int m = quarter * 32 + lane;
        const uint32_t tlane = (uint32_t)(quarter * 32) << 16;
        const int64_t col_a = (int64_t)tc.bi * kGT + m;
        float sxa = 0.f, sqa = 0.f, nmua = 0.f;
        if (col_a < a.f) {
            const double* c = a.cs + col_a * 12;
            sxa = (float)c[0];
            sqa = (float)c[1];
            nmua = -((float)c[9] * sxa);
        }
        const int64_t rows_left = a.n - r0;
        const int64_t full_steps = rows_left / kGK;
        const int n_full = full_steps <= 0 ? 0 : (full_steps >= nk ? nk : (int)full_steps);
        const uint32_t tbase = tmem + tlane + kPTmemA;
        for (int k = grp; k < nk; k += kPGroups) {
            const int rs = k % kPRawStages, as = k % kPAStages;
            if (!warp_wait(rfull0 + 8 * rs, (k / kPRawStages) & 1, a.err, 5, lane)) break;
            const unsigned char* raw = rawring + rs * kRawBox;
            Split8 xo0, qo0, xo1, qo1;
            if (k < n_full) {
                convert_a<false>(raw, m, 0, kGK, sxa, nmua, sqa, xo0, qo0);
                convert_a<false>(raw, m, 1, kGK, sxa, nmua, sqa, xo1, qo1);
            } else {
                const int64_t left = rows_left - (int64_t)k * kGK;
                const int valid = left <= 0 ? 0 : (int)left;
                convert_a<true>(raw, m, 0, valid, sxa, nmua, sqa, xo0, qo0);
                convert_a<true>(raw, m, 1, valid, sxa, nmua, sqa, xo1, qo1);
            }
            // the A stage must be free: the MMAs of step k - 4 have completed
            if (k >= kPAStages && !warp_wait(aempty0 + 8 * as, ((k / kPAStages) - 1) & 1, a.err, 6, lane)) break;
            tc_fence_after();
            const uint32_t ta = tbase + (uint32_t)(as * kPTmemAStride);
            tmem_st4(ta + 0, xo0.hi);
            tmem_st4(ta + 4, xo1.hi);
            tmem_st4(ta + 8, xo0.lo);
            tmem_st4(ta + 12, xo1.lo);
            tmem_st4(ta + 16, qo0.hi);
            tmem_st4(ta + 20, qo1.hi);
            tmem_st4(ta + 24, qo0.lo);
            tmem_st4(ta + 28, qo1.lo);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(afull0 + 8 * as);
                // the raw A tile has been consumed (its values are in the stores above)
                mbar_arrive(rempty0 + 8 * rs);
            }
        }
        if (grp < 2) {
            // groups 0 and 1 drain the accumulators: the two warps of a lane quarter take
            // alternate 32-column chunks
            const bool done = warp_wait(accum, 0, a.err, 3, lane);
            tc_fence_after();
            if (done && nk > 0) {
                float* out = a.partial + ((int64_t)blockIdx.y * a.n_tiles + blockIdx.x) * 3 * kGT * kGT;
                #pragma unroll 1
                for (int idx = grp; idx < 3 * kGT / 32; idx += 2) {
                    // partial [C | Q | W]: C at TMEM column 0, W at 128, Q at 256
                    const int gi = idx >> 2, cc = (idx & 3) * 32;
                    const uint32_t tcol = (gi == 0 ? kTmemCW : gi == 1 ? kTmemQ : kTmemCW + kGT) + (uint32_t)cc;
                    float tt[32];
                    tmem_ld32(tmem + tlane + tcol, tt);
                    float* op = out + (int64_t)(idx * 32) * kGT + m;
                    #pragma unroll
                    for (int c = 0; c < 32; ++c) op[(int64_t)c * kGT] = tt[c];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        if (lane == 0) mbar_wait(accum, 0, a.err, 7);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

// B planes of columns [c0, c0 + 8 gridDim.y) (< f_pad), rows [256 blockIdx.x, +256): warp w
// converts column c0 + 8 blockIdx.y + w, thread = 8 rows (one K half of one 16-row step),
// read as two float4 (a warp reads 1 KB of one column); columns at or beyond f and rows at
// or beyond n are zero.  The arithmetic is gram_fused_kernel's B-side conversion:
// b' = fma(v, s, -fl32(mean) s), b' (s_y ycen), v^2 s_q, with v = x or 1/safe(x), each split
// into hi and lo fp16 planes (order BH WBH BL WBL BQH BQL).  Layout: step-major, then
// 128-column block, then plane: the 16 rows of step t of column c = 128 J + m are 32 bytes at
// ((t * nb + J) * 6 + plane) * 2048 + m * 16 halves, K half h in 16-byte chunk
// h ^ ((m >> 2) & 1) (the 32-byte swizzle of a 128-row K-major tile whose rows are the
// columns), so the six tiles of one step and block are one contiguous 24 KB run.  The CTA's
// 6 planes x 16 steps x 8 columns go through shared memory so the stores are 256-byte runs.
template <bool kRecip>
__global__ void __launch_bounds__(256) gram_bplanes_kernel(const float* __restrict__ x, int64_t ld, int64_t n,
                                                           int64_t f, int64_t c0, int64_t f_pad,
                                                           const double* __restrict__ cs,
                                                           const float* __restrict__ ys, float eps,
                                                           __half* __restrict__ planes) {
    __shared__ uint4 stage[kBPlanes][16][8][2];   // [plane][step][column][chunk]: 24 KB
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t cb = c0 + (int64_t)blockIdx.y * 8;   // first column of this CTA
    const int64_t c = cb + w;
    const int64_t r = (int64_t)blockIdx.x * 256 + lane * 8;
    uint4 o[kBPlanes];
    #pragma unroll
    for (int p = 0; p < kBPlanes; ++p) o[p] = make_uint4(0, 0, 0, 0);
    if (c < f) {
        const float4 u0 = __ldg(reinterpret_cast<const float4*>(x + c * ld + r));
        const float4 u1 = __ldg(reinterpret_cast<const float4*>(x + c * ld + r + 4));
        const float4 y0 = __ldg(reinterpret_cast<const float4*>(ys + r));
        const float4 y1 = __ldg(reinterpret_cast<const float4*>(ys + r + 4));
        float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
        if (kRecip) {
            #pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = safe_recip(v[e], eps);
        }
        const double* cc = cs + c * 12;
        const float s = (float)cc[kRecip ? 3 : 0], sq = (float)cc[kRecip ? 4 : 1];
        const float mus = (float)cc[kRecip ? 5 : 9] * s;
        const uint64_t s2 = pk(s, s), nmu = pk(-mus, -mus), sq2 = pk(sq, sq);
        uint64_t v2[4], t2[4];
        #pragma unroll
        for (int p = 0; p < 4; ++p) {
            const uint64_t x2 = pk(v[2 * p], v[2 * p + 1]);
            v2[p] = fma2(x2, s2, nmu);
            t2[p] = mul2(mul2(x2, x2), sq2);
            const bool k0 = r + 2 * p < n, k1 = r + 2 * p + 1 < n;
            const float2 cv = upk(v2[p]), qv = upk(t2[p]);
            v2[p] = pk(k0 ? cv.x : 0.f, k1 ? cv.y : 0.f);
            t2[p] = pk(k0 ? qv.x : 0.f, k1 ? qv.y : 0.f);
        }
        Split8 b, w, q;
        split8(v2, b);
        split8(t2, q);
        v2[0] = mul2(v2[0], pk(y0.x, y0.y));
        v2[1] = mul2(v2[1], pk(y0.z, y0.w));
        v2[2] = mul2(v2[2], pk(y1.x, y1.y));
        v2[3] = mul2(v2[3], pk(y1.z, y1.w));
        split8(v2, w);
        o[0] = make_uint4(b.hi[0], b.hi[1], b.hi[2], b.hi[3]);
        o[1] = make_uint4(w.hi[0], w.hi[1], w.hi[2], w.hi[3]);
        o[2] = make_uint4(b.lo[0], b.lo[1], b.lo[2], b.lo[3]);
        o[3] = make_uint4(w.lo[0], w.lo[1], w.lo[2], w.lo[3]);
        o[4] = make_uint4(q.hi[0], q.hi[1], q.hi[2], q.hi[3]);
        o[5] = make_uint4(q.lo[0], q.lo[1], q.lo[2], q.lo[3]);
    }
    const int chunk = (lane & 1) ^ (int)((c >> 2) & 1);
    #pragma unroll
    for (int p = 0; p < kBPlanes; ++p) stage[p][lane >> 1][w][chunk] = o[p];
    __syncthreads();
    const int64_t nb = f_pad / kGT, t0 = (int64_t)blockIdx.x * 16, J = cb / kGT, m0 = cb % kGT;
    uint4* out = reinterpret_cast<uint4*>(planes);
    for (int q = threadIdx.x; q < kBPlanes * 16 * 16; q += 256) {
        const int p = q >> 8, st = (q >> 4) & 15, e = q & 15;   // e: column (e >> 1), chunk (e & 1)
        // in uint4: a 4 KB tile is 256, one column's step 2
        out[(((t0 + st) * nb + J) * kBPlanes + p) * 256 + m0 * 2 + e] = stage[p][st][e >> 1][e & 1];
    }
}

// ---- per-column statistics and scales -------------------------------------------

// Per column and row split: [0] min x, [1] max x, [2] sum g, [3] sum g^2, [4] sum g*ycen,
// [5] min g, [6] max g, [7] sum x, [8] sum x^2, [9] sum x*ycen
struct GramColPart {
    double v[10];
};

constexpr int kStatCols = 4;        // columns per CTA of the statistics pass
constexpr int kStatColsRecip = 2;   // ... when g = 1/safe(x) is accumulated too
constexpr int kMaxStatSplits = 64;  // row spans per column of the statistics pass

__device__ __forceinline__ double warp_sum(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// One 2048-row pass of the statistics kernel for one thread (two float4 runs per column).
// kMask: rows e of run u count only when e < valid_u (the rows left before n).
template <int kCB, bool kRecip, bool kMask>
__device__ __forceinline__ void stat_pass(const float4 (&xv)[kCB][2], const float4 (&yv)[2], int valid0, int valid1,
                                          float eps, float (&mn)[kCB], float (&mx)[kCB], float (&gmn)[kCB],
                                          float (&gmx)[kCB], double (&S)[kCB], double (&Q)[kCB], double (&W)[kCB],
                                          double (&G)[kCB], double (&GQ)[kCB], double (&GW)[kCB]) {
    #pragma unroll
    for (int c = 0; c < kCB; ++c) {
        float s1 = 0.f, q1 = 0.f, w1 = 0.f, g1 = 0.f, gq1 = 0.f, gw1 = 0.f;
        #pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float xs[4] = {xv[c][u].x, xv[c][u].y, xv[c][u].z, xv[c][u].w};
            const float ys[4] = {yv[u].x, yv[u].y, yv[u].z, yv[u].w};
            const int valid = u == 0 ? valid0 : valid1;
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
                const bool in = !kMask || e < valid;
                const float v = xs[e];
                s1 += v;
                q1 = fmaf(v, v, q1);
                w1 = fmaf(v, ys[e], w1);
                mn[c] = fminf(mn[c], in ? v : INFINITY);
                mx[c] = fmaxf(mx[c], in ? v : -INFINITY);
                if (kRecip) {
                    const float gv = in ? safe_recip(v, eps) : 0.f;
                    g1 += gv;
                    gq1 = fmaf(gv, gv, gq1);
                    gw1 = fmaf(gv, ys[e], gw1);
                    gmn[c] = fminf(gmn[c], in ? gv : INFINITY);
                    gmx[c] = fmaxf(gmx[c], in ? gv : -INFINITY);
                }
            }
        }
        S[c] += s1;
        Q[c] += q1;
        W[c] += w1;
        if (kRecip) {
            G[c] += g1;
            GQ[c] += gq1;
            GW[c] += gw1;
        }
    }
}

// One pass over the columns: the column sums the epilogue and the reconstruction need
// (sum x, sum x^2, sum x*ycen) and the ranges that set the operand scales, plus the same
// for g = 1/safe(x) when the divide group is scored (kRecip).  A CTA takes kCB columns and
// a row span; each thread reads float4 runs of 4 rows (rows up to ld exist: the padding is
// zero in x and ycen, which adds nothing to the sums, and is masked out of the ranges and
// of g).  Each thread adds its 8 rows of a pass in fp32 and the passes in fp64, in a fixed
// order, so the result does not depend on timing.
template <int kCB, bool kRecip>
__global__ void __launch_bounds__(256) gram_stats_kernel(const float* __restrict__ x, int64_t ld, int64_t n,
                                                         int64_t c_base, int64_t f, const float* __restrict__ ycen,
                                                         float eps, int64_t span, GramColPart* part) {
    // columns c_base + blockIdx.x * kCB + (0 .. kCB-1), those below f
    __shared__ double red[8][kCB][10];
    const int64_t c0 = c_base + (int64_t)blockIdx.x * kCB;
    const int s = blockIdx.y, splits = gridDim.y;
    const int64_t rb = (int64_t)s * span, re = min(rb + span, ld);   // span: a multiple of 2048
    float mn[kCB], mx[kCB], gmn[kCB], gmx[kCB];
    double S[kCB], Q[kCB], W[kCB], G[kCB], GQ[kCB], GW[kCB];
    #pragma unroll
    for (int c = 0; c < kCB; ++c) {
        mn[c] = gmn[c] = INFINITY;
        mx[c] = gmx[c] = -INFINITY;
        S[c] = Q[c] = W[c] = G[c] = GQ[c] = GW[c] = 0.0;
    }
    for (int64_t base = rb; base < re; base += 2048) {
        float4 yv[2], xv[kCB][2];
        #pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int64_t r = base + 1024 * u + 4 * threadIdx.x;
            const bool ok = r < re;
            yv[u] = ok ? __ldg(reinterpret_cast<const float4*>(ycen + r)) : make_float4(0.f, 0.f, 0.f, 0.f);
            #pragma unroll
            for (int c = 0; c < kCB; ++c)
                xv[c][u] = (ok && c0 + c < f) ? __ldg(reinterpret_cast<const float4*>(x + (c0 + c) * ld + r))
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (base + 2048 <= n) {
            stat_pass<kCB, kRecip, false>(xv, yv, 0, 0, eps, mn, mx, gmn, gmx, S, Q, W, G, GQ, GW);
        } else {
            // rows from n on are padding: masked out of the ranges and of g
            const int64_t left = n - (base + 4 * threadIdx.x);
            const int v0 = left <= 0 ? 0 : (left >= 4 ? 4 : (int)left);
            const int v1 = left <= 1024 ? 0 : (left >= 1028 ? 4 : (int)(left - 1024));
            stat_pass<kCB, kRecip, true>(xv, yv, v0, v1, eps, mn, mx, gmn, gmx, S, Q, W, G, GQ, GW);
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    #pragma unroll
    for (int c = 0; c < kCB; ++c) {
        const double v[10] = {(double)warp_min(mn[c]), (double)warp_max(mx[c]), warp_sum(G[c]), warp_sum(GQ[c]),
                              warp_sum(GW[c]), (double)warp_min(gmn[c]), (double)warp_max(gmx[c]), warp_sum(S[c]),
                              warp_sum(Q[c]), warp_sum(W[c])};
        if (lane == 0)
            for (int m = 0; m < 10; ++m) red[warp][c][m] = v[m];
    }
    __syncthreads();
    if (threadIdx.x < kCB * 10) {
        const int c = threadIdx.x / 10, m = threadIdx.x % 10;
        double acc = red[0][c][m];
        for (int w = 1; w < 8; ++w) {
            const double t = red[w][c][m];
            acc = (m == 0 || m == 5) ? fmin(acc, t) : (m == 1 || m == 6) ? fmax(acc, t) : acc + t;
        }
        if (c0 + c < f) part[(c0 + c) * splits + s].v[m] = acc;
    }
}

// Per-column scales and statistics of the operands:
//   cs[c*12 + 0..4]: s_x, s_q, s_w, s_g, s_gq (powers of two)
//   cs[c*12 + 5]: mean g rounded to fp32 (the value the operand conversion subtracts)
//   cs[c*12 + 6..8]: sum g, sum g^2, sum g*ycen
//   cs[c*12 + 9]: mean x rounded to fp32 (the value the operand conversion subtracts)
// and the column statistics the epilogue reads: colstats[c*4 + {0,1,2,3}] =
// {sum x, sum x^2, sum x*ycen, mean x}.
struct GramScaleArgs {
    const GramColPart* part;
    int splits;
    int64_t c_base, f, n;     // columns c_base .. f-1
    double* colstats;
    const unsigned* ycen_absmax;   // bits of max |ycen| (a non-negative float)
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

// s_y: the largest power of two with s_y * max|ycen| <= 1 (1 for a zero target)
__device__ __forceinline__ double ycen_scale(const unsigned* bits) {
    const float yabs = __uint_as_float(*bits);
    if (!(yabs > 0.0f) || !isfinite(yabs)) return 1.0;
    int e;
    frexp(1.0 / (double)yabs, &e);
    return ldexp(1.0, e - 1);
}

__global__ void gram_scale_kernel(GramScaleArgs a) {
    int64_t c = a.c_base + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= a.f) return;
    double mn = INFINITY, mx = -INFINITY, sg = 0, sgg = 0, sgy = 0, gmn = INFINITY, gmx = -INFINITY;
    double sx = 0, sxx = 0, sxy = 0;
    for (int s = 0; s < a.splits; ++s) {
        const GramColPart& p = a.part[c * a.splits + s];
        mn = fmin(mn, p.v[0]);
        mx = fmax(mx, p.v[1]);
        sg += p.v[2];
        sgg += p.v[3];
        sgy += p.v[4];
        gmn = fmin(gmn, p.v[5]);
        gmx = fmax(gmx, p.v[6]);
        sx += p.v[7];
        sxx += p.v[8];
        sxy += p.v[9];
    }
    const double n = (double)a.n;
    double* col = a.colstats + c * 4;
    col[0] = sx;
    col[1] = sxx;
    col[2] = sxy;
    col[3] = sx / n;
    const double mu = (double)(float)(sx / n);
    // the fp32 subtraction may round up by one ulp: a 2^-20 margin keeps |value| <= 2^14
    const double dev = fmax(fabs(mx - mu), fabs(mu - mn)) * (1.0 + 1e-6);
    double* o = a.cs + c * 12;
    o[0] = pow2_scale(dev);
    o[1] = pow2_scale(fmax(mx * mx, mn * mn) * (1.0 + 1e-6));
    o[2] = o[0] * ycen_scale(a.ycen_absmax);   // W operand = (s_x a') * (s_y ycen)
    o[9] = mu;
    if (a.recip) {
        const double mug = (double)(float)(sg / n);
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

// ys = ycen * s_y
__global__ void scale_rows_kernel(const float* __restrict__ v, int64_t n, const unsigned* absmax_bits,
                                  float* __restrict__ out) {
    const float s = (float)ycen_scale(absmax_bits);
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        out[r] = v[r] * s;
}

__global__ void absmax_kernel(const float* __restrict__ v, int64_t n, unsigned* out_bits) {
    float m = 0.0f;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(v[r]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(out_bits, __float_as_uint(m));  // non-negative floats order as uints
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
// Block (t, y): pairs q = 64 y .. 64 y + 63 of 64-tile t; the four 64-thread groups add
// the chunk partials of four consecutive chunk ranges, then group 0 adds the four range
// sums in range order (a fixed order: deterministic) and undoes scales and centring.
constexpr int kRedParts = 4;
__global__ void __launch_bounds__(256) gram_reduce_kernel(GramReduceArgs a) {
    __shared__ double red[3][kRedParts][64];
    const int t = blockIdx.x;
    const TileCoord tc = a.tiles64[t];
    const int I = tc.bi >> 1, J = tc.bj >> 1;
    const int t128 = a.lut[I * a.nb128 + J];
    const double n = (double)a.n;
    double* out = a.moments + (int64_t)t * 3 * kTilePairs;
    const int part = threadIdx.x >> 6;
    const int q = blockIdx.y * 64 + (threadIdx.x & 63);   // 0 .. 4095
    const int lj = q / kTile, li = q % kTile;
    const int e = li * kTile + lj;
    const int m = (tc.bi & 1) * kTile + li, nn = (tc.bj & 1) * kTile + lj;
    const int64_t i = (int64_t)tc.bi * kTile + li, j = (int64_t)tc.bj * kTile + lj;
    const bool live = t128 >= 0 && i < a.f && j < a.f;
    {
        double C = 0.0, Q = 0.0, W = 0.0;
        if (live) {
            const int per = (a.n_chunks + kRedParts - 1) / kRedParts;
            const int c0 = part * per, c1 = min(a.n_chunks, c0 + per);
            const float* p = a.partial + (int64_t)t128 * 3 * kGT * kGT + (int64_t)nn * kGT + m;
            const int64_t cstride = (int64_t)a.n_tiles128 * 3 * kGT * kGT;
            #pragma unroll 4
            for (int ch = c0; ch < c1; ++ch) {
                const float* pc = p + ch * cstride;
                C += (double)pc[0];
                Q += (double)pc[(int64_t)kGT * kGT];
                W += (double)pc[(int64_t)2 * kGT * kGT];
            }
        }
        red[0][part][threadIdx.x & 63] = C;
        red[1][part][threadIdx.x & 63] = Q;
        red[2][part][threadIdx.x & 63] = W;
    }
    __syncthreads();
    if (part != 0) return;
    double S1 = 0.0, Q = 0.0, S3 = 0.0;
    if (live) {
        double C = 0.0, W = 0.0;
        for (int r = 0; r < kRedParts; ++r) {
            C += red[0][r][threadIdx.x];
            Q += red[1][r][threadIdx.x];
            W += red[2][r][threadIdx.x];
        }
        const double* ci = a.cs + i * 12;
        const double* cj = a.cs + j * 12;
        const double mua = ci[9];                 // the mean the operand conversion subtracted (fp32)
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

bool make_x_map(CUtensorMap* map, const float* base, int64_t ld, int64_t f) {
    auto enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)ld, (cuuint64_t)f};
    cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(float)};
    cuuint32_t box[2] = {(cuuint32_t)kGK, (cuuint32_t)kGT};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
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

// The B-planes kernel is opt-in (GAFIME_GRAM_KERNEL=planes; =fused forces the fused kernel).
// Measured on the 2e6 x 2048 table it runs the Gram tiles in 92 ms against the fused
// kernel's 104 ms, but writing the planes costs 17 ms, so the fused kernel stays the
// default at every width.  kPlanesMinReuse (tiles per distinct B block) is the rule the
// default would use once the planes pay for themselves.
constexpr double kPlanesMinReuse = 1e30;

int gram_kernel_env() {
    static int env = -1;
    if (env < 0) {
        const char* v = getenv("GAFIME_GRAM_KERNEL");
        env = !v ? 0 : std::string(v) == "fused" ? 1 : std::string(v) == "planes" ? 2 : 0;
    }
    return env;
}

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

// Per-column state of one scoring call on the Gram path (statistics partials, operand
// scales and means, the scaled target, the error flag), independent of the tile set.
struct GramCols {
    GramColPart* colp;   // [f][kMaxStatSplits]
    double* cs;          // [f][12]
    float* ys;           // [ld]
    int* err;
    unsigned* absmax;
};

cudaError_t gram_cols(Bucket& b, GramCols& g) {
    const int64_t f = b.f, ld = b.ld;
    const size_t off_cs = ((size_t)f * kMaxStatSplits * sizeof(GramColPart) + 255) / 256 * 256;
    const size_t off_ys = (off_cs + (size_t)f * 12 * sizeof(double) + 255) / 256 * 256;
    const size_t off_err = (off_ys + (size_t)ld * sizeof(float) + 255) / 256 * 256;
    cudaError_t e = ensure(b.gram_cols, off_err + 256);
    if (e != cudaSuccess) return e;
    char* base = (char*)b.gram_cols.ptr;
    g.colp = (GramColPart*)base;
    g.cs = (double*)(base + off_cs);
    g.ys = (float*)(base + off_ys);
    g.err = (int*)(base + off_err);
    g.absmax = (unsigned*)(base + off_err + 64);
    return cudaSuccess;
}

cudaError_t gram_prep_target(Bucket& b, const ColumnStats& cs, cudaStream_t stream) {
    GramCols g;
    cudaError_t e = gram_cols(b, g);
    if (e != cudaSuccess) return e;
    KernelTimer timer(stream, GAFIME_KERNEL_GRAM_PREP);
    e = cudaMemsetAsync(g.absmax, 0, sizeof(unsigned), stream);
    if (e != cudaSuccess) return e;
    absmax_kernel<<<2 * b.sm_count, 256, 0, stream>>>(cs.d_ycen, b.ld, g.absmax);
    scale_rows_kernel<<<2 * b.sm_count, 256, 0, stream>>>(cs.d_ycen, b.ld, g.absmax, g.ys);
    return cudaGetLastError();
}

cudaError_t gram_prep_columns(Bucket& b, const ColumnStats& cs, bool recip, float eps, int64_t c0, int64_t c1,
                              cudaStream_t stream) {
    // one pass over columns [c0, c1): column sums (the epilogue's statistics) and ranges (and
    // the divide side's sums) -> power-of-two scales; no host round trip.  About 8 CTAs
    // per SM, row spans of whole 2048-row passes.
    if (c1 <= c0) return cudaSuccess;
    GramCols g;
    cudaError_t e = gram_cols(b, g);
    if (e != cudaSuccess) return e;
    const int64_t ld = b.ld, n = b.n;
    // the row spans follow from the whole matrix's column count, so a column's sums are the
    // same whichever range it is prepared in
    const int stat_cols = recip ? kStatColsRecip : kStatCols;
    const int64_t col_groups = (c1 - c0 + stat_cols - 1) / stat_cols;
    const int64_t all_groups = (b.f + stat_cols - 1) / stat_cols;
    int splits = (int)std::max<int64_t>(1, std::min<int64_t>((8 * (int64_t)b.sm_count + all_groups - 1) / all_groups,
                                                             (ld + 2047) / 2048));
    splits = std::min(splits, kMaxStatSplits);
    const int64_t span = ((ld + splits - 1) / splits + 2047) / 2048 * 2048;
    KernelTimer timer(stream, GAFIME_KERNEL_GRAM_PREP);
    if (recip)
        gram_stats_kernel<kStatColsRecip, true><<<dim3((unsigned)col_groups, (unsigned)splits), 256, 0, stream>>>(
            cs.d_x, ld, n, c0, c1, cs.d_ycen, eps, span, g.colp);
    else
        gram_stats_kernel<kStatCols, false><<<dim3((unsigned)col_groups, (unsigned)splits), 256, 0, stream>>>(
            cs.d_x, ld, n, c0, c1, cs.d_ycen, eps, span, g.colp);
    GramScaleArgs sa;
    sa.part = g.colp;
    sa.splits = splits;
    sa.c_base = c0;
    sa.f = c1;
    sa.n = n;
    sa.colstats = const_cast<double*>(cs.d_col);
    sa.ycen_absmax = g.absmax;
    sa.recip = recip ? 1 : 0;
    sa.cs = g.cs;
    gram_scale_kernel<<<(unsigned)((c1 - c0 + 127) / 128), 128, 0, stream>>>(sa);
    return cudaGetLastError();
}

int64_t gram_chunk_rows(const Bucket& b) {
    // row chunks: <= max_chunk_rows() rows, about four CTAs per SM over the whole matrix's
    // 128-tiles.  The chunk follows from the matrix alone, never from the tiles of one shard
    // or one streamed set, so every pair's fp32 partial sums cover the same rows whichever
    // shard scores it: a sharded top-k is bit-identical to the single-GPU one.
    const int64_t ld = b.ld;
    const int64_t nb128 = (b.f + kGT - 1) / kGT;
    const int64_t all_tiles = std::max<int64_t>(1, nb128 * (nb128 + 1) / 2);
    const int64_t want = std::max<int64_t>(1, (4 * (int64_t)b.sm_count + all_tiles - 1) / all_tiles);
    int64_t chunk = (ld + want - 1) / want;
    chunk = std::min<int64_t>(max_chunk_rows(), std::max<int64_t>(1024, chunk));
    return (chunk + kRowPad - 1) / kRowPad * kRowPad;
}

bool gram_use_planes(const Bucket& b, const std::vector<TileCoord>& tiles64) {
    const int env = gram_kernel_env();
    if (env != 0) return env == 2;
    const int nb128 = (int)((b.f + kGT - 1) / kGT);
    std::vector<char> seen((size_t)nb128 * nb128, 0), bcol((size_t)nb128, 0);
    int tiles = 0, bblocks = 0;
    for (const TileCoord& t : tiles64) {
        const int I = t.bi >> 1, J = t.bj >> 1;
        if (!seen[(size_t)I * nb128 + J]) {
            seen[(size_t)I * nb128 + J] = 1;
            ++tiles;
        }
        if (!bcol[(size_t)J]) {
            bcol[(size_t)J] = 1;
            ++bblocks;
        }
    }
    return bblocks > 0 && (double)tiles / bblocks >= kPlanesMinReuse;
}

cudaError_t launch_gram_moments(Bucket& b, const ColumnStats& cs, const TileCoord* d_tiles64,
                                const std::vector<TileCoord>& tiles64, bool recip, float eps,
                                double* d_moments, cudaStream_t stream, int* host_err, int prep_mode,
                                int64_t chunk_rows, int use_planes) {
    if (host_err) *host_err = 0;
    const int64_t f = b.f, ld = b.ld, n = b.n;
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
    const bool planes = use_planes < 0 ? gram_use_planes(b, tiles64) : use_planes != 0;
    const int64_t chunk = chunk_rows > 0 ? chunk_rows : gram_chunk_rows(b);
    const int n_chunks = (int)((ld + chunk - 1) / chunk);

    // scratch of this tile set: partial | lut | tiles128; the per-column state (scales, scaled
    // target, error flag) lives in its own buffer, shared by both moment groups of a call and
    // by every tile set of a streamed call, and the B planes in theirs
    size_t part_bytes = (size_t)n_chunks * nt * 3 * kGT * kGT * sizeof(float);
    size_t off_lut = (part_bytes + 255) / 256 * 256;
    size_t off_t128 = (off_lut + lut.size() * sizeof(int) + 255) / 256 * 256;
    size_t total = (off_t128 + t128.size() * sizeof(TileCoord) + 255) / 256 * 256;
    cudaError_t e = ensure(b.gram, total);
    if (e != cudaSuccess) return e;
    const int64_t f_pad = (int64_t)nb128 * kGT;
    if (planes) {
        e = ensure(b.gram_planes, (size_t)kBPlanes * f_pad * ld * sizeof(__half));
        if (e != cudaSuccess) return e;
    }
    GramCols gc;
    e = gram_cols(b, gc);
    if (e != cudaSuccess) return e;
    char* base = (char*)b.gram.ptr;
    float* partial = (float*)base;
    int* d_lut = (int*)(base + off_lut);
    TileCoord* d_t128 = (TileCoord*)(base + off_t128);
    double* d_cs = gc.cs;
    float* d_ys = gc.ys;
    int* d_err = gc.err;

    e = cudaMemcpyAsync(d_lut, lut.data(), lut.size() * sizeof(int), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_t128, t128.data(), t128.size() * sizeof(TileCoord), cudaMemcpyHostToDevice, stream);
    // the flag only (absmax follows at +64); with host_err null the caller clears and reads it
    if (e == cudaSuccess && host_err) e = cudaMemsetAsync(d_err, 0, 64, stream);
    if (e != cudaSuccess) return e;

    if (prep_mode != GRAM_PREP_DONE) {
        e = gram_prep_target(b, cs, stream);
        if (e == cudaSuccess)
        {
            // only the 128-column blocks this call's tiles read (a shard of many GPUs needs a
            // few of them); runs of consecutive blocks go in one launch
            std::vector<char> used((size_t)nb128, 0);
            for (const TileCoord& t : t128) used[(size_t)t.bi] = used[(size_t)t.bj] = 1;
            for (int B0 = 0; B0 < nb128 && e == cudaSuccess;) {
                if (!used[(size_t)B0]) { ++B0; continue; }
                int B1 = B0;
                while (B1 < nb128 && used[(size_t)B1]) ++B1;
                e = gram_prep_columns(b, cs, recip || prep_mode == GRAM_PREP_BOTH, eps, (int64_t)B0 * kGT,
                                      std::min<int64_t>(f, (int64_t)B1 * kGT), stream);
                B0 = B1;
            }
        }
        if (e != cudaSuccess) return e;
    }

    CUtensorMap xmap;
    if (!make_x_map(&xmap, cs.d_x, ld, f)) return cudaErrorInvalidValue;
    if (planes) {
        // the B planes of the blocks this set reads as B (runs of consecutive blocks per launch)
        __half* d_planes = (__half*)b.gram_planes.ptr;
        std::vector<char> bused((size_t)nb128, 0);
        for (const TileCoord& t : t128) bused[(size_t)t.bj] = 1;
        {
            KernelTimer timer(stream, GAFIME_KERNEL_GRAM_PREP);
            for (int B0 = 0; B0 < nb128;) {
                if (!bused[(size_t)B0]) { ++B0; continue; }
                int B1 = B0;
                while (B1 < nb128 && bused[(size_t)B1]) ++B1;
                // grid: 256-row slabs x 8-column groups (at most 32768 groups per launch)
                for (int64_t c0 = (int64_t)B0 * kGT; c0 < (int64_t)B1 * kGT; c0 += 8 * 32768) {
                    const int64_t cols = std::min<int64_t>(8 * 32768, (int64_t)B1 * kGT - c0);
                    const dim3 grid((unsigned)(ld / 256), (unsigned)(cols / 8));
                    if (recip)
                        gram_bplanes_kernel<true><<<grid, 256, 0, stream>>>(cs.d_x, ld, n, f, c0, f_pad, d_cs, d_ys,
                                                                           eps, d_planes);
                    else
                        gram_bplanes_kernel<false><<<grid, 256, 0, stream>>>(cs.d_x, ld, n, f, c0, f_pad, d_cs, d_ys,
                                                                            eps, d_planes);
                }
                B0 = B1;
            }
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        PlanesArgs pa;
        pa.nb = f_pad / kGT;
        pa.planes = d_planes;
        pa.tiles = d_t128;
        pa.n_tiles = nt;
        pa.chunk_rows = chunk;
        pa.rows = ld;
        pa.n = n;
        pa.f = f;
        pa.cs = d_cs;
        pa.partial = partial;
        pa.err = d_err;
        e = cudaFuncSetAttribute(gram_planes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPlanesSmem);
        if (e != cudaSuccess) return e;
        KernelTimer timer(stream, GAFIME_KERNEL_GRAM_TC);
        gram_planes_kernel<<<dim3((unsigned)nt, (unsigned)n_chunks), kGramThreads, kPlanesSmem, stream>>>(xmap, pa);
        e = cudaGetLastError();
    } else {
        GramArgs ga;
        ga.tiles = d_t128;
        ga.n_tiles = nt;
        ga.chunk_rows = chunk;
        ga.rows = ld;
        ga.n = n;
        ga.f = f;
        ga.ys = d_ys;
        ga.cs = d_cs;
        ga.recip = recip ? 1 : 0;
        ga.eps = eps;
        ga.partial = partial;
        ga.err = d_err;
        e = cudaFuncSetAttribute(gram_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGramSmem);
        if (e != cudaSuccess) return e;
        KernelTimer timer(stream, GAFIME_KERNEL_GRAM_TC);
        gram_fused_kernel<<<dim3((unsigned)nt, (unsigned)n_chunks), kGramThreads, kGramSmem, stream>>>(xmap, ga);
        e = cudaGetLastError();
    }
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
        gram_reduce_kernel<<<dim3((unsigned)tiles64.size(), kTilePairs / 64), 256, 0, stream>>>(ra);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess || !host_err) return e;
    int h_err = 0;
    e = cudaMemcpyAsync(&h_err, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    *host_err = h_err;
    return e;
}

cudaError_t gram_error_reset(Bucket& b, cudaStream_t stream) {
    GramCols g;
    cudaError_t e = gram_cols(b, g);
    return e == cudaSuccess ? cudaMemsetAsync(g.err, 0, 64, stream) : e;
}

const double* gram_col_state(Bucket& b) {
    GramCols g;
    return gram_cols(b, g) == cudaSuccess ? g.cs : nullptr;
}

cudaError_t gram_error_read(Bucket& b, cudaStream_t stream, int* host_err) {
    GramCols g;
    cudaError_t e = gram_cols(b, g);
    int h = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h, g.err, sizeof(int), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    *host_err = h;
    return e;
}

}  // namespace gafime
