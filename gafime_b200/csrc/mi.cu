// mi.cu -- all-pairs mutual information with equal-width bins.
//
// Semantics of gafime_core.score_combos for 2-combos (gafime_core.cpp:531-618):
//   x_r = (a_r - mean_a) * (b_r - mean_b) in fp64           (gafime_core.cpp:571-577)
//   y bins:  build_bins(y, bins)  min/max equal width        (gafime_core.cpp:200-226)
//   x bins:  (int)((x - xmin) * bins / (xmax - xmin)), clamped   (gafime_core.cpp:277-304)
//   MI = sum_{bx,by} p log(p / (p_x p_y)), natural log       (gafime_core.cpp:316-332)
//   MI = 0 when xmin == xmax or y is constant.
// With center = 0 the interaction is the kernel-API x = fl32(a op b)
// (cpu_backend.cpp:87-103) and the same binning applies.
//
// Device plan (per call):
//   y codes : y-bin of every row, remapped to the U bins that occur (exact: bins no row
//             falls in contribute nothing);
//   class copy: the feature columns are copied with their rows grouped by y code, so every
//             row split below holds rows of one y class only and a pair's histogram for it
//             is one row of `bins` counters (the joint histogram is order-free);
//   pass 1  : per-pair min / max of x over row splits, merged with 64-bit integer
//             atomics on an order-preserving key (deterministic);
//   pass 2  : each thread owns one pair and a private x histogram for the split's
//             class in shared memory; split results merge into the joint histogram with
//             integer atomics;
//   finish  : MI per pair in fp64 in the reference's summation order, then the same
//             bitonic top-k as the Pearson epilogue.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <vector>

#include "engine.h"
#include "select.cuh"

namespace gafime {

namespace {

constexpr int kMiRows = 64;                  // rows per shared-memory chunk
constexpr int64_t kMiMaxSplitRows = 32768;   // rows per split at most

__device__ __forceinline__ long long dkey(double v) {
    long long b = __double_as_longlong(v);
    return b >= 0 ? b : (b ^ 0x7FFFFFFFFFFFFFFFLL);
}
__device__ __forceinline__ double dval(long long k) {
    return __longlong_as_double(k >= 0 ? k : (k ^ 0x7FFFFFFFFFFFFFFFLL));
}

// Rows [r0, r1) of the class-grouped copy, all of y class u
struct MiSplit {
    int64_t r0, r1;
    int u, pad;
};

struct MiArgs {
    const float* xs;          // class-grouped copy of the feature columns, [f][lds]
    int64_t lds, f;
    const double* colstats;   // mean at [c*4 + 3]
    const TileCoord* tiles;
    int n_tiles;
    int op;
    float eps;
    const MiSplit* splits;
    long long* mm;            // [n_tiles][4096][2] keys: min, max
    int bins, U;
    unsigned* hist;           // [n_tiles][4096][bins * U]
};

// Column stride of the staged operand blocks: four rows load as one 16-byte vector, and
// the 16 columns a warp reads start in distinct bank groups.
template <typename V>
struct Stage {
    static constexpr int kStride = sizeof(V) == 8 ? kMiRows + 2 : kMiRows + 4;
};

template <int OP>
__device__ __forceinline__ double combine_t(double a, double b, double eps) {
    if (OP == GAFIME_INTERACT_ADD) return a + b;
    if (OP == GAFIME_INTERACT_SUB) return a - b;
    if (OP == GAFIME_INTERACT_DIV) return a / (fabs(b) < eps ? copysign(eps, b) : b);
    return __dmul_rn(a, b);
}
template <int OP>
__device__ __forceinline__ float combine_t(float a, float b, float eps) {
    if (OP == GAFIME_INTERACT_ADD) return a + b;
    if (OP == GAFIME_INTERACT_SUB) return a - b;
    if (OP == GAFIME_INTERACT_DIV) return a / (fabsf(b) < eps ? copysignf(eps, b) : b);
    return __fmul_rn(a, b);
}

// A staged value the fp32 pre-filter of pass 1 cannot bound: nonzero with magnitude outside
// [2^-60, 2^60] (its fp32 copy or a product of two could leave the normal fp32 range)
__device__ __forceinline__ int out_of_filter_range(double v) {
    const double m = fabs(v);
    return m != 0.0 && (m < 0x1p-60 || m > 0x1p60);
}

// Four consecutive staged rows of one column
__device__ __forceinline__ void load4(const double* p, double v[4]) {
    const double2 a = *reinterpret_cast<const double2*>(p);
    const double2 b = *reinterpret_cast<const double2*>(p + 2);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void load4(const float* p, float v[4]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}

// One CTA: one TS x TS block of pairs inside a 64 x 64 tile, one row split.  The
// interaction operator is a template argument so the row loop holds no branch on it.
template <int TS, int PASS, bool CENTRED, int OP>
__global__ void __launch_bounds__(TS * TS) mi_pass_kernel(MiArgs a) {
    using V = typename std::conditional<CENTRED, double, float>::type;
    constexpr int SUBS = 64 / TS;
    constexpr int kS = Stage<V>::kStride;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    V* As = reinterpret_cast<V*>(smem_raw);                  // [TS][kS]: column-major rows
    V* Bs = As + TS * kS;                                    // [TS][kS]
    unsigned* hs = reinterpret_cast<unsigned*>(Bs + TS * kS);  // [warps][bins][32 lanes]
    // Pass 1 of the centred product also stages fp32 copies of the operands: the min / max
    // scan runs on fp32 products and falls back to the exact fp64 products only for rows
    // that could move the current minimum or maximum (see the bound below).
    constexpr bool kFilter = PASS == 1 && CENTRED && OP == GAFIME_INTERACT_MULT;
    constexpr int kSf = kMiRows + 4;
    float* Af = reinterpret_cast<float*>(Bs + TS * kS);       // [TS][kSf] (kFilter only)
    float* Bf = Af + TS * kSf;

    const int t = blockIdx.x / (SUBS * SUBS), sub = blockIdx.x % (SUBS * SUBS);
    const int si = sub / SUBS, sj = sub % SUBS;
    const TileCoord tc = a.tiles[t];
    if (tc.bi == tc.bj && si > sj) return;
    const int64_t i0 = (int64_t)tc.bi * 64 + si * TS, j0 = (int64_t)tc.bj * 64 + sj * TS;
    if (i0 >= a.f || j0 >= a.f) return;
    const int tid = threadIdx.x;
    // a warp holds 4 x 8 pairs: its operand loads touch 4 A columns and 8 B columns, one
    // wavefront each per four rows
    constexpr int kWarpsPerBand = TS / 8;
    const int warp = tid >> 5, lane = tid & 31;
    const int li = (warp / kWarpsPerBand) * 4 + (lane >> 3), lj = (warp % kWarpsPerBand) * 8 + (lane & 7);
    const int64_t i = i0 + li, j = j0 + lj;
    const bool valid = (i < j) && (j < a.f);
    const int e = (si * TS + li) * 64 + (sj * TS + lj);
    long long* mm = a.mm + ((int64_t)t * kTilePairs + e) * 2;

    const MiSplit sp = a.splits[blockIdx.y];
    const int64_t r0 = sp.r0, r1 = sp.r1;

    double mn[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
    double mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    double xmin = 0.0, scale = 0.0;
    bool live = valid;
    // Each thread's private x histogram: counter c of lane l at word c * 32 + l of its warp's
    // block, so the lanes of a warp always hit 32 distinct banks.  Counts go in with shared
    // atomics whose result nobody waits for: consecutive rows of a thread never stall on a
    // load-add-store round trip through the same counter.
    unsigned* h = hs + (tid >> 5) * (a.bins * 32) + (tid & 31);
    const int top = a.bins - 1;
    if (PASS == 2) {
        for (int c = 0; c < a.bins; ++c) h[c * 32] = 0;
        if (valid) {
            xmin = dval(mm[0]);
            double xmax = dval(mm[1]);
            live = xmax != xmin;
            scale = (double)a.bins / (xmax - xmin);
        }
    }
    const V* ap = As + li * kS;
    const V* bp = Bs + lj * kS;
    const V eps = (V)a.eps;

    // The raw values of the next chunk are loaded into registers while this chunk is
    // computed, so the global-load latency hides behind the row loop.
    constexpr int kPer = kMiRows / TS;  // staged values per thread and operand
    float pa[kPer], pb[kPer];
    auto fetch = [&](int64_t rb) {
        const int rows = (int)std::min<int64_t>(kMiRows, r1 - rb);
        #pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int q = tid + u * TS * TS, col = q / kMiRows, row = q % kMiRows;
            const int64_t ca = i0 + col, cb = j0 + col;
            pa[u] = (row < rows && ca < a.f) ? a.xs[ca * a.lds + rb + row] : 0.f;
            pb[u] = (row < rows && cb < a.f) ? a.xs[cb * a.lds + rb + row] : 0.f;
        }
    };
    if (r0 < r1) fetch(r0);
    for (int64_t rb = r0; rb < r1; rb += kMiRows) {
        const int rows = (int)std::min<int64_t>(kMiRows, r1 - rb);
        int unsafe = 0;
        __syncthreads();
        #pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int q = tid + u * TS * TS, col = q / kMiRows, row = q % kMiRows;
            const int64_t ca = i0 + col, cb = j0 + col;
            V va, vb;
            if (CENTRED) {
                va = ca < a.f ? (V)((double)pa[u] - a.colstats[ca * 4 + 3]) : (V)0;
                vb = cb < a.f ? (V)((double)pb[u] - a.colstats[cb * 4 + 3]) : (V)0;
            } else {
                va = (V)pa[u];
                vb = (V)pb[u];
            }
            As[col * kS + row] = va;
            Bs[col * kS + row] = vb;
            if (kFilter) {
                Af[col * kSf + row] = (float)va;
                Bf[col * kSf + row] = (float)vb;
                unsafe |= out_of_filter_range((double)va) | out_of_filter_range((double)vb);
            }
        }
        const bool exact_chunk = kFilter ? __syncthreads_or(unsafe) != 0 : true;
        if (!kFilter) __syncthreads();
        if (rb + kMiRows < r1) fetch(rb + kMiRows);
        if (!live) continue;
        if (kFilter) {
            // Every staged |value| is 0 or in [2^-60, 2^60], so a32 = a(1+e1), b32 = b(1+e2)
            // and p32 = a32 b32 (1+e3), |e| <= 2^-24, with no underflow or overflow: p32 is
            // within 2^-22 |p| of the exact product p.  A row with p > max has
            // p32 >= max - 2^-22 |max| (either sign), hence p32 >= thr_hi below (margin 2^-20,
            // rounded down), so rows below both thresholds cannot move the min or the max.
            const float* afp = Af + li * kSf;
            const float* bfp = Bf + lj * kSf;
            float thr_hi = __double2float_rd(mx[0] - fabs(mx[0]) * 0x1p-20);
            float thr_lo = __double2float_ru(mn[0] + fabs(mn[0]) * 0x1p-20);
            int r = 0;
            for (; r + 8 <= rows; r += 8) {
                // eight rows: the extremes of their fp32 products against the thresholds
                // (no product is NaN in a chunk inside the bound's range)
                float fa[8], fb[8];
                load4(afp + r, fa);
                load4(afp + r + 4, fa + 4);
                load4(bfp + r, fb);
                load4(bfp + r + 4, fb + 4);
                float p[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) p[u] = __fmul_rn(fa[u], fb[u]);
                const float hi = fmaxf(fmaxf(fmaxf(p[0], p[1]), fmaxf(p[2], p[3])),
                                       fmaxf(fmaxf(p[4], p[5]), fmaxf(p[6], p[7])));
                const float lo = fminf(fminf(fminf(p[0], p[1]), fminf(p[2], p[3])),
                                       fminf(fminf(p[4], p[5]), fminf(p[6], p[7])));
                // a chunk outside the bound's range: every row exact
                if (exact_chunk || !(hi < thr_hi) || !(lo > thr_lo)) {
                    #pragma unroll
                    for (int h = 0; h < 8; h += 4) {
                        V av[4], bv[4];
                        load4(ap + r + h, av);
                        load4(bp + r + h, bv);
                        #pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const double xv = (double)combine_t<OP>(av[u], bv[u], eps);
                            mn[0] = xv < mn[0] ? xv : mn[0];
                            mx[0] = xv > mx[0] ? xv : mx[0];
                        }
                    }
                    thr_hi = __double2float_rd(mx[0] - fabs(mx[0]) * 0x1p-20);
                    thr_lo = __double2float_ru(mn[0] + fabs(mn[0]) * 0x1p-20);
                }
            }
            for (; r < rows; ++r) {
                const double xv = (double)combine_t<OP>(ap[r], bp[r], eps);
                mn[0] = xv < mn[0] ? xv : mn[0];
                mx[0] = xv > mx[0] ? xv : mx[0];
            }
            continue;
        }
        // four rows per iteration: products and bins are independent chains; only the
        // histogram updates (which may hit the same counter) stay in row order
        int r = 0;
        for (; r + 4 <= rows; r += 4) {
            V av[4], bv[4];
            load4(ap + r, av);
            load4(bp + r, bv);
            double xv[4];
            #pragma unroll
            for (int u = 0; u < 4; ++u) xv[u] = (double)combine_t<OP>(av[u], bv[u], eps);
            if (PASS == 1) {
                #pragma unroll
                for (int u = 0; u < 4; ++u) {
                    mn[u] = xv[u] < mn[u] ? xv[u] : mn[u];
                    mx[u] = xv[u] > mx[u] ? xv[u] : mx[u];
                }
            } else {
                // xv >= xmin holds exactly (xmin is the minimum of these same values), so the
                // bin index is never negative; xv = xmax can land on bins and is clamped
                #pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int xb = (int)((xv[u] - xmin) * scale);
                    atomicAdd(&h[(xb < top ? xb : top) * 32], 1u);
                }
            }
        }
        for (; r < rows; ++r) {
            const double xv = (double)combine_t<OP>(ap[r], bp[r], eps);
            if (PASS == 1) {
                mn[0] = xv < mn[0] ? xv : mn[0];
                mx[0] = xv > mx[0] ? xv : mx[0];
            } else {
                const int xb = (int)((xv - xmin) * scale);
                atomicAdd(&h[(xb < top ? xb : top) * 32], 1u);
            }
        }
    }
    if (!valid) return;
    if (PASS == 1) {
        if (r1 > r0) {
            const double lo = fmin(fmin(mn[0], mn[1]), fmin(mn[2], mn[3]));
            const double hi = fmax(fmax(mx[0], mx[1]), fmax(mx[2], mx[3]));
            atomicMin(&mm[0], dkey(lo));
            atomicMax(&mm[1], dkey(hi));
        }
    } else if (live) {
        unsigned* g = a.hist + ((int64_t)t * kTilePairs + e) * (a.bins * a.U) + sp.u;
        for (int c = 0; c < a.bins; ++c)
            if (h[c * 32]) atomicAdd(&g[c * a.U], h[c * 32]);
    }
}

// Copy the feature columns with their rows grouped by y code: row r goes to the next free
// slot of its class (cursor[u] starts at the class's first row).  Rows of one class land in
// arbitrary order, which nothing downstream depends on (histograms and min / max are
// order-free).  Each warp claims one contiguous run per class it holds, so the stores of a
// warp fall into at most a few runs per column.
__global__ void __launch_bounds__(256) class_scatter_kernel(const float* __restrict__ x, int64_t ld,
                                                            int64_t f, int64_t n,
                                                            const uint8_t* __restrict__ ycode,
                                                            unsigned long long* cursor, float* xs,
                                                            int64_t lds) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t base = warp * 32; base < n; base += warps * 32) {
        const int64_t r = base + lane;
        const bool in = r < n;
        const unsigned active = __ballot_sync(0xffffffffu, in);
        if (!in) continue;
        const int code = ycode[r];
        const unsigned same = __match_any_sync(active, code);
        const int leader = __ffs(same) - 1;
        unsigned long long first = 0;
        if (lane == leader) first = atomicAdd(&cursor[code], (unsigned long long)__popc(same));
        first = __shfl_sync(same, first, leader);
        const int64_t dest = (int64_t)first + __popc(same & ((1u << lane) - 1u));
        for (int64_t c = 0; c < f; ++c) xs[c * lds + dest] = x[c * ld + r];
    }
}

__global__ void mm_init_kernel(long long* mm, int64_t count) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < count;
         q += (int64_t)gridDim.x * blockDim.x) {
        mm[2 * q] = 0x7FFFFFFFFFFFFFFFLL;
        mm[2 * q + 1] = (long long)0x8000000000000000ULL;
    }
}

// ---- y bins -----------------------------------------------------------------

__global__ void ymm_kernel(const float* y, int64_t n, long long* ymm) {
    double mn = INFINITY, mx = -INFINITY;
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n;
         r += (int64_t)gridDim.x * blockDim.x) {
        double v = y[r];
        mn = v < mn ? v : mn;
        mx = v > mx ? v : mx;
    }
    if (mn <= mx) {
        atomicMin(&ymm[0], dkey(mn));
        atomicMax(&ymm[1], dkey(mx));
    }
}

__device__ __forceinline__ int ybin_of(double v, double ymin, double yscale, int bins) {
    int b = (int)((v - ymin) * yscale);
    return b < 0 ? 0 : (b >= bins ? bins - 1 : b);
}

__global__ void ycount_kernel(const float* y, int64_t n, const long long* ymm, int bins,
                              unsigned* counts) {
    double ymin = dval(ymm[0]), ymax = dval(ymm[1]);
    if (!(ymax > ymin)) return;
    double ys = (double)bins / (ymax - ymin);
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n;
         r += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(&counts[ybin_of(y[r], ymin, ys, bins)], 1u);
}

// counts[bins] -> map[bins] (compact code or 255) and meta = {U, ready}
__global__ void ymap_kernel(const unsigned* counts, const long long* ymm, int bins, int* map,
                            int* meta) {
    double ymin = dval(ymm[0]), ymax = dval(ymm[1]);
    int ready = ymax > ymin;
    int u = 0;
    for (int b = 0; b < bins; ++b) map[b] = (ready && counts[b]) ? u++ : 255;
    meta[0] = u;
    meta[1] = ready;
}

__global__ void ycode_kernel(const float* y, int64_t n, const long long* ymm, int bins,
                             const int* map, uint8_t* ycode) {
    double ymin = dval(ymm[0]), ymax = dval(ymm[1]);
    double ys = (double)bins / (ymax - ymin);
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n;
         r += (int64_t)gridDim.x * blockDim.x)
        ycode[r] = (uint8_t)map[ybin_of(y[r], ymin, ys, bins)];
}

// ---- finish: MI per pair + top-k ----------------------------------------------

struct MiFinishArgs {
    const TileCoord* tiles;
    int n_tiles;
    int64_t f, n;
    const long long* mm;
    const unsigned* hist;
    const unsigned* ycounts;  // [bins] rows per y bin (p_y of the reference)
    const int* map;           // [bins] compact codes
    int bins, U, ready;
    int k_pad;
    Cand* cands;
    double* all_scores;
};

__global__ void __launch_bounds__(256) mi_finish_kernel(MiFinishArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Cand* s = reinterpret_cast<Cand*>(smem_raw);
    __shared__ double py[256];
    const int t = blockIdx.x;
    const TileCoord tc = a.tiles[t];
    for (int b = threadIdx.x; b < a.bins; b += blockDim.x) {
        int c = a.map[b];
        if (c != 255) py[c] = (double)a.ycounts[b];
    }
    __syncthreads();
    const double inv_total = 1.0 / (double)a.n;
    const double inv_total_sq = inv_total * inv_total;
    for (int e = threadIdx.x; e < kTilePairs; e += blockDim.x) {
        int li = e / kTile, lj = e % kTile;
        int64_t i = (int64_t)tc.bi * kTile + li, j = (int64_t)tc.bj * kTile + lj;
        Cand c;
        c.pad = 0;
        if (i < j && j < a.f) {
            double mi = 0.0;
            const long long* mm = a.mm + ((int64_t)t * kTilePairs + e) * 2;
            if (a.ready && mm[0] != mm[1]) {
                const unsigned* h = a.hist + ((int64_t)t * kTilePairs + e) * (a.bins * a.U);
                for (int bx = 0; bx < a.bins; ++bx) {
                    double px = 0.0;
                    for (int u = 0; u < a.U; ++u) px += (double)h[bx * a.U + u];
                    if (px == 0.0) continue;
                    for (int u = 0; u < a.U; ++u) {
                        double count = (double)h[bx * a.U + u];
                        if (count <= 0.0) continue;
                        double p = count * inv_total;
                        double expected = (px * py[u]) * inv_total_sq;
                        if (expected > 0.0) mi += p * log(p / expected);
                    }
                }
            }
            c.score = mi;
            c.pid = (uint32_t)(i * a.f + j);
            if (a.all_scores) a.all_scores[i * a.f - i * (i + 1) / 2 + (j - i - 1)] = mi;
        } else {
            c.score = 0.0;
            c.pid = kNoPair;
        }
        s[e] = c;
    }
    if (a.cands == nullptr) return;
    __syncthreads();
    bitonic_sort(s, kTilePairs);
    Cand* out = a.cands + (int64_t)t * a.k_pad;
    for (int e = threadIdx.x; e < a.k_pad; e += blockDim.x) out[e] = s[e];
}

template <int TS, int PASS, bool CENTRED, int OP>
cudaError_t launch_pass(const MiArgs& a, int splits, cudaStream_t stream) {
    using V = typename std::conditional<CENTRED, double, float>::type;
    size_t smem = 2 * sizeof(V) * TS * Stage<V>::kStride;
    if (PASS == 1 && CENTRED && OP == GAFIME_INTERACT_MULT) smem += 2 * sizeof(float) * TS * (kMiRows + 4);
    if (PASS == 2) smem += (size_t)((TS * TS + 31) / 32) * a.bins * 32 * sizeof(unsigned);
    auto kern = mi_pass_kernel<TS, PASS, CENTRED, OP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)(a.n_tiles * (64 / TS) * (64 / TS)), (unsigned)splits);
    kern<<<grid, TS * TS, smem, stream>>>(a);
    return cudaGetLastError();
}

template <int TS, bool CENTRED, int OP>
cudaError_t run_passes_op(const MiArgs& a, int splits, cudaStream_t stream) {
    cudaError_t e;
    {
        KernelTimer timer(stream, GAFIME_KERNEL_MI_PASS1);
        e = launch_pass<TS, 1, CENTRED, OP>(a, splits, stream);
    }
    if (e == cudaSuccess) {
        KernelTimer timer(stream, GAFIME_KERNEL_MI_PASS2);
        e = launch_pass<TS, 2, CENTRED, OP>(a, splits, stream);
    }
    return e;
}

template <int TS, bool CENTRED>
cudaError_t run_passes(const MiArgs& a, int splits, cudaStream_t stream) {
    switch (a.op) {
        case GAFIME_INTERACT_ADD: return run_passes_op<TS, CENTRED, GAFIME_INTERACT_ADD>(a, splits, stream);
        case GAFIME_INTERACT_SUB: return run_passes_op<TS, CENTRED, GAFIME_INTERACT_SUB>(a, splits, stream);
        case GAFIME_INTERACT_DIV: return run_passes_op<TS, CENTRED, GAFIME_INTERACT_DIV>(a, splits, stream);
        default: return run_passes_op<TS, CENTRED, GAFIME_INTERACT_MULT>(a, splits, stream);
    }
}

}  // namespace

// y bins of the target: equal-width bins (gafime_core.cpp:200-226) remapped to the
// U bins that occur.  One small host sync learns U.
struct YBins {
    long long* ymm;     // [2] order-preserving keys of min / max y
    unsigned* counts;   // [256] rows per y bin (p_y of the reference)
    int* map;           // [256] compact code per bin, 255 when unused
    uint8_t* ycode;     // [n] compact code per row
    int U = 1, ready = 0;
    unsigned hcounts[256];  // host copy of counts
};

cudaError_t prepare_ybins(Bucket& b, int bins, YBins& yb, cudaStream_t stream) {
    size_t off_ymm = 0, off_counts = 64, off_map = off_counts + 256 * 4, off_meta = off_map + 256 * 4;
    size_t off_ycode = (off_meta + 64 + 255) / 256 * 256;
    size_t bytes = off_ycode + ((size_t)b.ld + 255) / 256 * 256;
    cudaError_t e = ensure(b.mi, bytes);
    if (e != cudaSuccess) return e;
    char* base = (char*)b.mi.ptr;
    yb.ymm = (long long*)(base + off_ymm);
    yb.counts = (unsigned*)(base + off_counts);
    yb.map = (int*)(base + off_map);
    int* meta = (int*)(base + off_meta);
    yb.ycode = (uint8_t*)(base + off_ycode);
    const float* y = b.d_data + b.f * b.ld;
    long long init[2] = {0x7FFFFFFFFFFFFFFFLL, (long long)0x8000000000000000ULL};
    e = cudaMemcpyAsync(yb.ymm, init, sizeof(init), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(yb.counts, 0, 256 * 4, stream);
    if (e != cudaSuccess) return e;
    ymm_kernel<<<2 * b.sm_count, 256, 0, stream>>>(y, b.n, yb.ymm);
    ycount_kernel<<<2 * b.sm_count, 256, 0, stream>>>(y, b.n, yb.ymm, bins, yb.counts);
    ymap_kernel<<<1, 1, 0, stream>>>(yb.counts, yb.ymm, bins, yb.map, meta);
    int hmeta[2] = {0, 0};
    e = cudaMemcpyAsync(hmeta, meta, sizeof(hmeta), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(yb.hcounts, yb.counts, sizeof(yb.hcounts), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return e;
    yb.U = std::max(1, hmeta[0]);
    yb.ready = hmeta[1];
    if (yb.ready) ycode_kernel<<<2 * b.sm_count, 256, 0, stream>>>(y, b.n, yb.ymm, bins, yb.map, yb.ycode);
    return cudaGetLastError();
}

cudaError_t launch_mi_scores(Bucket& b, const ColumnStats& cs, bool centred, int op, float div_eps,
                             int mi_bins, const TileCoord* d_tiles, int n_tiles, int k_pad,
                             Cand* cands, double* all_scores, cudaStream_t stream) {
    const int bins = mi_bins;
    YBins yb;
    cudaError_t e = prepare_ybins(b, bins, yb, stream);
    if (e != cudaSuccess) return e;
    const int U = yb.U, ready = yb.ready;
    long long* mm = nullptr;
    unsigned* hist = nullptr;
    // tiles per batch: the joint histograms of one batch stay under 2 GiB
    const size_t tile_bytes = (size_t)kTilePairs * (bins * U * sizeof(unsigned) + 2 * sizeof(long long));
    const int batch = (int)std::max<size_t>(1, std::min<size_t>((size_t)n_tiles, ((size_t)2 << 30) / tile_bytes));
    e = ensure(b.mi_mm, (size_t)batch * kTilePairs * 2 * sizeof(long long));
    if (e == cudaSuccess) e = ensure(b.mi_hist, (size_t)batch * kTilePairs * bins * U * sizeof(unsigned));
    if (e != cudaSuccess) return e;
    mm = (long long*)b.mi_mm.ptr;
    hist = (unsigned*)b.mi_hist.ptr;

    MiArgs a;
    a.f = b.f;
    a.colstats = cs.d_col;
    a.op = op;
    a.eps = div_eps;
    a.mm = mm;
    a.bins = bins;
    a.U = U;
    a.hist = hist;
    int n_splits = 0;
    if (ready) {
        // rows per split: at most 32768, fewer while the grid would hold
        // under 4 CTAs per SM
        int64_t per = std::min<int64_t>(kMiMaxSplitRows, (b.n + 1) / 2 + kMiRows);
        per = std::max<int64_t>(kMiRows, (per + kMiRows - 1) / kMiRows * kMiRows);
        auto count_splits = [&](int64_t p) {
            int64_t s = 0;
            for (int u = 0, c = 0; c < bins; ++c)
                if (yb.hcounts[c]) { s += ((int64_t)yb.hcounts[c] + p - 1) / p; ++u; }
            return s;
        };
        const int64_t ctas_per_split = (int64_t)std::min(batch, n_tiles) * 16;
        while (count_splits(per) * ctas_per_split < 4 * b.sm_count && per > 4 * kMiRows)
            per = std::max<int64_t>(kMiRows, (per / 2 + kMiRows - 1) / kMiRows * kMiRows);
        std::vector<MiSplit> host;
        std::vector<unsigned long long> first;
        int64_t off = 0;
        for (int c = 0; c < bins; ++c) {
            if (!yb.hcounts[c]) continue;
            const int u = (int)first.size();
            first.push_back((unsigned long long)off);
            for (int64_t r = off; r < off + yb.hcounts[c]; r += per)
                host.push_back(MiSplit{r, std::min<int64_t>(r + per, off + yb.hcounts[c]), u, 0});
            off += yb.hcounts[c];
        }
        if (host.size() > 65535 || (int)first.size() != U || off != b.n) return cudaErrorInvalidValue;
        n_splits = (int)host.size();
        // cursor[256] | splits[n_splits]
        e = ensure(b.mi_split, 256 * sizeof(unsigned long long) + host.size() * sizeof(MiSplit));
        if (e != cudaSuccess) return e;
        unsigned long long* cursor = (unsigned long long*)b.mi_split.ptr;
        MiSplit* d_splits = (MiSplit*)(cursor + 256);
        const int64_t lds = (b.n + 31) / 32 * 32;
        e = ensure(b.mi_xs, (size_t)b.f * lds * sizeof(float));
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(cursor, first.data(), first.size() * sizeof(unsigned long long),
                                cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(d_splits, host.data(), host.size() * sizeof(MiSplit), cudaMemcpyHostToDevice,
                                stream);
        if (e != cudaSuccess) return e;
        {
            KernelTimer timer(stream, GAFIME_KERNEL_MI_CLASS_COPY);
            class_scatter_kernel<<<4 * b.sm_count, 256, 0, stream>>>(b.d_data, b.ld, b.f, b.n, yb.ycode, cursor,
                                                                     (float*)b.mi_xs.ptr, lds);
        }
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        a.xs = (const float*)b.mi_xs.ptr;
        a.lds = lds;
        a.splits = d_splits;
    }

    MiFinishArgs fa;
    fa.f = b.f;
    fa.n = b.n;
    fa.mm = mm;
    fa.hist = hist;
    fa.ycounts = yb.counts;
    fa.map = yb.map;
    fa.bins = bins;
    fa.U = U;
    fa.ready = ready;
    fa.k_pad = k_pad;
    fa.all_scores = all_scores;
    const size_t fsmem = sizeof(Cand) * kTilePairs;
    e = cudaFuncSetAttribute(mi_finish_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fsmem);
    if (e != cudaSuccess) return e;
    for (int t0 = 0; t0 < n_tiles; t0 += batch) {
        const int nt = std::min(batch, n_tiles - t0);
        mm_init_kernel<<<2 * b.sm_count, 256, 0, stream>>>(mm, (int64_t)nt * kTilePairs);
        e = cudaMemsetAsync(hist, 0, (size_t)nt * kTilePairs * bins * U * sizeof(unsigned), stream);
        if (e != cudaSuccess) return e;
        if (ready) {
            a.tiles = d_tiles + t0;
            a.n_tiles = nt;
            // 16 x 16 pairs per CTA while their histograms fit in shared memory (bins <= 192),
            // else 8 x 8
            if (bins <= 192)
                e = centred ? run_passes<16, true>(a, n_splits, stream) : run_passes<16, false>(a, n_splits, stream);
            else
                e = centred ? run_passes<8, true>(a, n_splits, stream) : run_passes<8, false>(a, n_splits, stream);
            if (e != cudaSuccess) return e;
        }
        fa.tiles = d_tiles + t0;
        fa.n_tiles = nt;
        fa.cands = cands ? cands + (int64_t)t0 * k_pad : nullptr;
        KernelTimer timer(stream, GAFIME_KERNEL_MI_FINISH);
        mi_finish_kernel<<<nt, 256, fsmem, stream>>>(fa);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ---- unary mutual information (one raw column against y) -------------------

namespace {

__global__ void __launch_bounds__(256) unary_mm_kernel(const float* __restrict__ x, int64_t ld,
                                                       int64_t n, int64_t rps, long long* mm) {
    __shared__ double smn[256], smx[256];
    const int c = blockIdx.x;
    const int64_t r0 = (int64_t)blockIdx.y * rps, r1 = std::min<int64_t>(r0 + rps, n);
    double mn = INFINITY, mx = -INFINITY;
    for (int64_t r = r0 + threadIdx.x; r < r1; r += 256) {
        double v = x[(int64_t)c * ld + r];
        mn = v < mn ? v : mn;
        mx = v > mx ? v : mx;
    }
    smn[threadIdx.x] = mn;
    smx[threadIdx.x] = mx;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            smn[threadIdx.x] = fmin(smn[threadIdx.x], smn[threadIdx.x + s]);
            smx[threadIdx.x] = fmax(smx[threadIdx.x], smx[threadIdx.x + s]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0 && r1 > r0) {
        atomicMin(&mm[2 * c], dkey(smn[0]));
        atomicMax(&mm[2 * c + 1], dkey(smx[0]));
    }
}

// kShared: count in a shared-memory copy of the column's joint histogram, else straight
// into global memory (joint histograms over 48K counters)
template <bool kShared>
__global__ void __launch_bounds__(256) unary_hist_kernel(const float* __restrict__ x, int64_t ld,
                                                         int64_t n, int64_t rps, const long long* mm,
                                                         const uint8_t* ycode, int bins, int U,
                                                         unsigned* hist) {
    extern __shared__ unsigned hsh[];  // [bins * U]
    const int c = blockIdx.x;
    unsigned* h = kShared ? hsh : hist + (int64_t)c * bins * U;
    if (kShared) {
        for (int q = threadIdx.x; q < bins * U; q += 256) h[q] = 0;
        __syncthreads();
    }
    const double xmin = dval(mm[2 * c]), xmax = dval(mm[2 * c + 1]);
    if (xmax != xmin) {
        const double scale = (double)bins / (xmax - xmin);
        const int64_t r0 = (int64_t)blockIdx.y * rps, r1 = std::min<int64_t>(r0 + rps, n);
        for (int64_t r = r0 + threadIdx.x; r < r1; r += 256) {
            int xb = (int)(((double)x[(int64_t)c * ld + r] - xmin) * scale);
            xb = xb < 0 ? 0 : (xb >= bins ? bins - 1 : xb);
            atomicAdd(&h[xb * U + ycode[r]], 1u);
        }
    }
    if (!kShared) return;
    __syncthreads();
    for (int q = threadIdx.x; q < bins * U; q += 256)
        if (h[q]) atomicAdd(&hist[(int64_t)c * bins * U + q], h[q]);
}

__global__ void unary_finish_kernel(int64_t f, int64_t n, const long long* mm, const unsigned* hist,
                                    const unsigned* ycounts, const int* map, int bins, int U,
                                    int ready, double* out) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= f) return;
    double py[256];
    for (int b = 0; b < bins; ++b)
        if (map[b] != 255) py[map[b]] = (double)ycounts[b];
    const double inv_total = 1.0 / (double)n, inv_total_sq = inv_total * inv_total;
    double mi = 0.0;
    if (ready && mm[2 * c] != mm[2 * c + 1]) {
        const unsigned* hc = hist + c * bins * U;
        for (int bx = 0; bx < bins; ++bx) {
            double px = 0.0;
            for (int u = 0; u < U; ++u) px += (double)hc[bx * U + u];
            if (px == 0.0) continue;
            for (int u = 0; u < U; ++u) {
                double count = (double)hc[bx * U + u];
                if (count <= 0.0) continue;
                double p = count * inv_total;
                double expected = (px * py[u]) * inv_total_sq;
                if (expected > 0.0) mi += p * log(p / expected);
            }
        }
    }
    out[c] = mi;
}

}  // namespace

cudaError_t launch_mi_unary(Bucket& b, int mi_bins, double* d_out, cudaStream_t stream) {
    YBins yb;
    cudaError_t e = prepare_ybins(b, mi_bins, yb, stream);
    if (e != cudaSuccess) return e;
    const int U = yb.U, bins = mi_bins;
    e = ensure(b.mi_mm, (size_t)b.f * 2 * sizeof(long long));
    if (e == cudaSuccess) e = ensure(b.mi_hist, (size_t)b.f * bins * U * sizeof(unsigned));
    if (e != cudaSuccess) return e;
    long long* mm = (long long*)b.mi_mm.ptr;
    unsigned* hist = (unsigned*)b.mi_hist.ptr;
    mm_init_kernel<<<(unsigned)((b.f + 255) / 256), 256, 0, stream>>>(mm, b.f);
    e = cudaMemsetAsync(hist, 0, (size_t)b.f * bins * U * sizeof(unsigned), stream);
    if (e != cudaSuccess) return e;
    if (yb.ready) {
        int splits = (int)std::max<int64_t>(1, std::min<int64_t>((4 * b.sm_count + b.f - 1) / b.f,
                                                                 (b.n + 16383) / 16384));
        int64_t rps = (b.n + splits - 1) / splits;
        dim3 grid((unsigned)b.f, (unsigned)splits);
        unary_mm_kernel<<<grid, 256, 0, stream>>>(b.d_data, b.ld, b.n, rps, mm);
        const size_t smem = (size_t)bins * U * sizeof(unsigned);
        if (smem <= 192 * 1024) {
            e = cudaFuncSetAttribute(unary_hist_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem);
            if (e != cudaSuccess) return e;
            unary_hist_kernel<true><<<grid, 256, smem, stream>>>(b.d_data, b.ld, b.n, rps, mm, yb.ycode, bins,
                                                                 U, hist);
        } else {
            unary_hist_kernel<false><<<grid, 256, 0, stream>>>(b.d_data, b.ld, b.n, rps, mm, yb.ycode, bins, U,
                                                               hist);
        }
    }
    unary_finish_kernel<<<(unsigned)((b.f + 127) / 128), 128, 0, stream>>>(
        b.f, b.n, mm, hist, yb.counts, yb.map, bins, U, yb.ready, d_out);
    return cudaGetLastError();
}

// ---- mutual information with quantile bins on the interaction -------------------------
//
// No counterpart in the reference, which bins equal-width only (gafime_core.cpp:200-226).
// Definition (restated in the oracle, which is the only check of it): the cut points of a
// pair are the order statistics t_b = sorted[floor(b n / bins)], b = 1 .. bins-1, of its n
// interaction values x; the bin of x is the number of cut points t_b <= x (ties share a bin,
// repeated cut points leave bins empty); a constant interaction scores 0.  y is binned
// equal-width as in the reference, and the MI sum is mi_finish_kernel's.
// Device plan, per batch of pairs: the interaction of every row as an order-preserving 64-bit
// key of its fp64 value (-0 made +0, so equal values have equal keys); one exact device
// radix sort per pair; the cut keys read at the ranks; then one pass over the unsorted keys
// bins each row by binary search among the cut keys into a joint histogram (shared-memory
// counters per CTA, added into the pair's histogram), and the MI per pair.

namespace {

constexpr int kQRows = 4096;   // rows per CTA of the binning pass

__device__ __forceinline__ unsigned long long okey(double v) {
    v = v + 0.0;   // -0 -> +0
    const unsigned long long u = (unsigned long long)__double_as_longlong(v);
    return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}

struct QArgs {
    const float* x;            // bucket matrix (raw), ld rows per column
    int64_t ld, n;
    const double* colstats;    // mean at [c*4 + 3]
    const int2* pairs;         // [batch] (i, j)
    int centred, op;
    float eps;
    unsigned long long* keys;  // [batch][n]
};

template <int OP>
__device__ __forceinline__ double q_interaction(float a, float b, double ma, double mb, int centred, float eps) {
    if (centred) return combine_t<OP>((double)a - ma, (double)b - mb, (double)eps);
    return (double)combine_t<OP>(a, b, eps);
}

// grid (ceil(n / 256), batch): keys of pair blockIdx.y
template <int OP>
__global__ void __launch_bounds__(256) q_keys_kernel(QArgs a) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.n) return;
    const int2 pr = a.pairs[blockIdx.y];
    const double ma = a.centred ? a.colstats[(int64_t)pr.x * 4 + 3] : 0.0;
    const double mb = a.centred ? a.colstats[(int64_t)pr.y * 4 + 3] : 0.0;
    const double v = q_interaction<OP>(a.x[(int64_t)pr.x * a.ld + r], a.x[(int64_t)pr.y * a.ld + r], ma, mb,
                                       a.centred, a.eps);
    a.keys[(int64_t)blockIdx.y * a.n + r] = okey(v);
}

// one thread per (pair, cut): cut keys t_b = sorted[floor(b n / bins)], and whether the pair
// is constant (sorted[0] == sorted[n - 1]) in cut slot bins - 1
__global__ void q_cuts_kernel(const unsigned long long* sorted, int64_t n, int bins, int batch,
                              unsigned long long* cuts) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= batch * bins) return;
    const int p = t / bins, b = t % bins;
    const unsigned long long* s = sorted + (int64_t)p * n;
    if (b == 0)
        cuts[(int64_t)p * bins + bins - 1] = s[0] == s[n - 1] ? 1ull : 0ull;
    else
        cuts[(int64_t)p * bins + b - 1] = s[(int64_t)b * n / bins];
}

// grid (ceil(n / kQRows), batch): joint histogram [bins][U] of pair blockIdx.y, counts added
// into hist[p] with integer atomics (order-free)
__global__ void __launch_bounds__(256) q_hist_kernel(const unsigned long long* keys, int64_t n,
                                                     const uint8_t* __restrict__ ycode,
                                                     const unsigned long long* cuts, int bins, int U,
                                                     unsigned* hist) {
    extern __shared__ unsigned qsm[];
    unsigned long long* cut = reinterpret_cast<unsigned long long*>(qsm);   // [bins - 1]
    unsigned* h = qsm + 2 * bins;                                          // [bins][U]
    const int p = blockIdx.y;
    for (int b = threadIdx.x; b < bins - 1; b += blockDim.x) cut[b] = cuts[(int64_t)p * bins + b];
    for (int c = threadIdx.x; c < bins * U; c += blockDim.x) h[c] = 0;
    __syncthreads();
    const unsigned long long* kp = keys + (int64_t)p * n;
    const int64_t r0 = (int64_t)blockIdx.x * kQRows, r1 = min(r0 + kQRows, n);
    for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
        const unsigned long long k = kp[r];
        int lo = 0, hi = bins - 1;   // number of cut keys <= k
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (cut[mid] <= k) lo = mid + 1; else hi = mid;
        }
        atomicAdd(&h[lo * U + ycode[r]], 1u);
    }
    __syncthreads();
    unsigned* g = hist + (int64_t)p * bins * U;
    for (int c = threadIdx.x; c < bins * U; c += blockDim.x)
        if (h[c]) atomicAdd(&g[c], h[c]);
}

// one thread per pair: MI in fp64, the summation order of mi_finish_kernel
__global__ void q_mi_kernel(const unsigned* hist, const unsigned long long* cuts, const unsigned* ycounts,
                            const int* map, int bins, int U, int ready, int64_t n, int batch, const int64_t* slot,
                            double* scores) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= batch) return;
    double py[256];
    for (int b = 0; b < bins; ++b) {
        const int c = map[b];
        if (c != 255) py[c] = (double)ycounts[b];
    }
    double mi = 0.0;
    if (ready && cuts[(int64_t)p * bins + bins - 1] == 0ull) {
        const double inv_total = 1.0 / (double)n, inv_total_sq = inv_total * inv_total;
        const unsigned* h = hist + (int64_t)p * bins * U;
        for (int bx = 0; bx < bins; ++bx) {
            double px = 0.0;
            for (int u = 0; u < U; ++u) px += (double)h[bx * U + u];
            if (px == 0.0) continue;
            for (int u = 0; u < U; ++u) {
                const double count = (double)h[bx * U + u];
                if (count <= 0.0) continue;
                const double pr = count * inv_total;
                const double expected = (px * py[u]) * inv_total_sq;
                if (expected > 0.0) mi += pr * log(pr / expected);
            }
        }
    }
    scores[slot[p]] = mi;   // the pair's place in the tile layout
}

// per-tile candidate lists from a dense score array [tile][kTilePairs] (the MI finish's
// ranking: bitonic top-k of the tile), and every score in triangle order when asked
__global__ void __launch_bounds__(256) q_lists_kernel(const double* scores, const TileCoord* tiles, int64_t f,
                                                      int k_pad, Cand* cands, double* all_scores) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Cand* s = reinterpret_cast<Cand*>(smem_raw);
    const int t = blockIdx.x;
    const TileCoord tc = tiles[t];
    for (int e = threadIdx.x; e < kTilePairs; e += blockDim.x) {
        const int64_t i = (int64_t)tc.bi * kTile + e / kTile, j = (int64_t)tc.bj * kTile + e % kTile;
        Cand c;
        c.pad = 0;
        if (i < j && j < f) {
            c.score = scores[(int64_t)t * kTilePairs + e];
            c.pid = (uint32_t)(i * f + j);
            if (all_scores) all_scores[i * f - i * (i + 1) / 2 + (j - i - 1)] = c.score;
        } else {
            c.score = 0.0;
            c.pid = kNoPair;
        }
        s[e] = c;
    }
    if (cands == nullptr) return;
    __syncthreads();
    bitonic_sort(s, kTilePairs);
    Cand* out = cands + (int64_t)t * k_pad;
    for (int e = threadIdx.x; e < k_pad; e += blockDim.x) out[e] = s[e];
}

}  // namespace

cudaError_t launch_mi_quantile(Bucket& b, const ColumnStats& cs, bool centred, int op, float div_eps, int mi_bins,
                               const std::vector<TileCoord>& tiles, const TileCoord* d_tiles, int k_pad,
                               Cand* cands, double* all_scores, cudaStream_t stream) {
    const int bins = mi_bins;
    const int n_tiles = (int)tiles.size();
    if (n_tiles == 0) return cudaSuccess;
    YBins yb;
    cudaError_t e = prepare_ybins(b, bins, yb, stream);
    if (e != cudaSuccess) return e;
    const int U = yb.U;
    if ((size_t)bins * U * sizeof(unsigned) + 2 * (size_t)bins * sizeof(unsigned) > 160 * 1024)
        return cudaErrorInvalidValue;   // the joint histogram of a CTA must fit in shared memory
    const int64_t n = b.n, f = b.f;
    // the pairs of the tiles, in tile-major order (pair q = tile * kTilePairs + e)
    std::vector<int2> pairs;
    std::vector<int64_t> slot;
    for (int t = 0; t < n_tiles; ++t)
        for (int e2 = 0; e2 < kTilePairs; ++e2) {
            const int64_t i = (int64_t)tiles[t].bi * kTile + e2 / kTile, j = (int64_t)tiles[t].bj * kTile + e2 % kTile;
            if (i < j && j < f) {
                pairs.push_back(make_int2((int)i, (int)j));
                slot.push_back((int64_t)t * kTilePairs + e2);
            }
        }
    const int64_t P = (int64_t)pairs.size();
    // pairs per batch: keys (two copies) under ~3 GiB, at most 65535 (grid.y)
    const int64_t batch = std::max<int64_t>(1, std::min<int64_t>({P, 65535, ((int64_t)3 << 30) / (16 * n)}));
    size_t temp_bytes = 0;
    cub::DeviceRadixSort::SortKeys(nullptr, temp_bytes, (const unsigned long long*)nullptr,
                                   (unsigned long long*)nullptr, (int)n);
    const size_t off_keys2 = ((size_t)batch * n * 8 + 255) / 256 * 256;
    const size_t off_temp = off_keys2 + ((size_t)batch * n * 8 + 255) / 256 * 256;
    const size_t off_cuts = off_temp + (temp_bytes + 255) / 256 * 256;
    const size_t off_hist = off_cuts + ((size_t)batch * bins * 8 + 255) / 256 * 256;
    const size_t off_scores = off_hist + ((size_t)batch * bins * U * 4 + 255) / 256 * 256;
    const size_t off_pairs = off_scores + ((size_t)n_tiles * kTilePairs * 8 + 255) / 256 * 256;
    const size_t off_slot = off_pairs + ((size_t)P * sizeof(int2) + 255) / 256 * 256;
    const size_t total = off_slot + (size_t)P * sizeof(int64_t);
    e = ensure(b.rank, total);
    if (e != cudaSuccess) return e;
    char* base = (char*)b.rank.ptr;
    unsigned long long* keys = (unsigned long long*)base;
    unsigned long long* keys2 = (unsigned long long*)(base + off_keys2);
    void* temp = base + off_temp;
    unsigned long long* cuts = (unsigned long long*)(base + off_cuts);
    unsigned* hist = (unsigned*)(base + off_hist);
    double* scores = (double*)(base + off_scores);
    int2* d_pairs = (int2*)(base + off_pairs);
    int64_t* d_slot = (int64_t*)(base + off_slot);
    e = cudaMemcpyAsync(d_pairs, pairs.data(), (size_t)P * sizeof(int2), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_slot, slot.data(), (size_t)P * sizeof(int64_t), cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(scores, 0, (size_t)n_tiles * kTilePairs * 8, stream);
    if (e != cudaSuccess) return e;
    const size_t hsmem = (size_t)bins * U * sizeof(unsigned) + 2 * (size_t)bins * sizeof(unsigned);
    e = cudaFuncSetAttribute(q_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hsmem);
    if (e != cudaSuccess) return e;
    for (int64_t p0 = 0; p0 < P; p0 += batch) {
        const int nb = (int)std::min<int64_t>(batch, P - p0);
        QArgs qa;
        qa.x = b.d_data;
        qa.ld = b.ld;
        qa.n = n;
        qa.colstats = cs.d_col;
        qa.pairs = d_pairs + p0;
        qa.centred = centred ? 1 : 0;
        qa.op = op;
        qa.eps = div_eps;
        qa.keys = keys;
        {
            KernelTimer timer(stream, GAFIME_KERNEL_MI_PASS1);
            const dim3 grid((unsigned)((n + 255) / 256), (unsigned)nb);
            switch (op) {
                case GAFIME_INTERACT_ADD: q_keys_kernel<GAFIME_INTERACT_ADD><<<grid, 256, 0, stream>>>(qa); break;
                case GAFIME_INTERACT_SUB: q_keys_kernel<GAFIME_INTERACT_SUB><<<grid, 256, 0, stream>>>(qa); break;
                case GAFIME_INTERACT_DIV: q_keys_kernel<GAFIME_INTERACT_DIV><<<grid, 256, 0, stream>>>(qa); break;
                default: q_keys_kernel<GAFIME_INTERACT_MULT><<<grid, 256, 0, stream>>>(qa);
            }
            e = cudaGetLastError();
            for (int q = 0; q < nb && e == cudaSuccess; ++q) {
                size_t tb = temp_bytes;
                e = cub::DeviceRadixSort::SortKeys(temp, tb, keys + (int64_t)q * n, keys2 + (int64_t)q * n, (int)n, 0,
                                                   64, stream);
            }
        }
        if (e != cudaSuccess) return e;
        q_cuts_kernel<<<(unsigned)((nb * bins + 255) / 256), 256, 0, stream>>>(keys2, n, bins, nb, cuts);
        e = cudaMemsetAsync(hist, 0, (size_t)nb * bins * U * 4, stream);
        if (e != cudaSuccess) return e;
        {
            KernelTimer timer(stream, GAFIME_KERNEL_MI_PASS2);
            if (yb.ready)
                q_hist_kernel<<<dim3((unsigned)((n + kQRows - 1) / kQRows), (unsigned)nb), 256, hsmem, stream>>>(
                    keys, n, yb.ycode, cuts, bins, U, hist);
        }
        q_mi_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, stream>>>(hist, cuts, yb.counts, yb.map, bins, U,
                                                                      yb.ready, n, nb, d_slot + p0, scores);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    const size_t lsmem = sizeof(Cand) * kTilePairs;
    e = cudaFuncSetAttribute(q_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsmem);
    if (e != cudaSuccess) return e;
    KernelTimer timer(stream, GAFIME_KERNEL_MI_FINISH);
    q_lists_kernel<<<n_tiles, 256, lsmem, stream>>>(scores, d_tiles, f, k_pad, cands, all_scores);
    return cudaGetLastError();
}

}  // namespace gafime
