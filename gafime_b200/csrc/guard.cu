// guard.cu -- accuracy guard of the Pearson epilogue and the exact re-score of the pairs
// it flags.
//
// The pair moments come from fp32 accumulations (tensor-core Gram tiles of 2-term fp16
// operands, or fp32 runs on the CUDA cores) that are exact enough for every pair whose
// interaction is well conditioned.  Two kinds of pair are not:
//   * S2 = sum x^2 is accumulated without centring, so var_x = S2 - S1^2/n inherits S2's
//     rounding magnified by the pair's conditioning S2 / (n var_x) (columns far from zero);
//   * on the Gram path S1 = sum a*g(b) is rebuilt from a Gram of centred columns, whose
//     rounding is on the scale of the columns' spreads, sqrt(n) sd_a sd_g: a product tiny
//     against both of its columns loses its variance to it.
// guard_kernel estimates, per pair and operator, the rounding of n var_x from what the
// epilogue holds (S1, S2, the columns' sums and squares):
//     err = c (S2 | Qa + Qb)  +  2 |S1| e1 / n + e1^2 / n        (multiply / divide)
//     err = c (Qa + Qb)       +  2 e1                             (add / subtract)
//     e1  = c sqrt(n) sd_a sd_g   (Gram path only)
// with c = 1e-6 (about four times the rounding a numerical model of the Gram path shows),
// and flags the pair when err > 1e-4 * n var_x (a collapsed or negative variance is always
// flagged unless the estimate is zero).  Flagged pairs go to a device list that
// rescore_kernel works through: it forms x = fl32(a op b) per row and sums x, x^2 and x*y in
// fp64, which is the reference's own arithmetic (src/cpu/cpu_backend.cpp:87-103,274-293),
// and writes the Pearson of those sums (native_cuda_backend.py:471-486) as the pair's
// score.  The epilogue then takes that score for every flagged pair.  Data that flags
// nothing pays one read of the moments and an empty launch.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "engine.h"

namespace gafime {

namespace {

constexpr double kGuardC = 1e-6;    // relative rounding per accumulated term (calibrated)
constexpr double kGuardTau = 1e-4;  // flag when the estimate exceeds this share of n var_x
constexpr int kGuardThreads = 256;
constexpr int kRescoreThreads = 256;

__device__ __forceinline__ double col_sd(double s, double q, double n) {
    const double m = s / n;
    const double v = q / n - m * m;
    return v > 0.0 ? sqrt(v) : 0.0;
}

// Grid (n_tiles, kTilePairs / 256, n_ops): one thread per pair e of tile t for operator o.
__global__ void __launch_bounds__(kGuardThreads) guard_kernel(GuardArgs a) {
    const int t = blockIdx.x, oi = blockIdx.z;
    const int e = blockIdx.y * kGuardThreads + threadIdx.x;
    const int op = a.op[oi], splits = a.splits[oi];
    const TileCoord tc = a.tiles[t];
    const int64_t i = (int64_t)tc.bi * kTile + e / kTile, j = (int64_t)tc.bj * kTile + e % kTile;
    const double n = a.ystats[0];
    bool flag = false;
    if (i < j && j < a.f && n > 1.0) {
        const double* moments = a.moments[oi];
        double S1 = 0.0, S2 = 0.0;
        for (int sp = 0; sp < splits; ++sp) {
            const double* m = moments + ((int64_t)sp * a.n_tiles + t) * 3 * kTilePairs;
            S1 += m[e];
            S2 += m[kTilePairs + e];
        }
        const double* ci = a.colstats + i * 4;
        const double* cj = a.colstats + j * 4;
        double e1 = 0.0;
        if (a.gram) {
            // spread of the B side: g = 1/safe(b) for divide (the Gram column state), b otherwise
            const double sd_g = op == GAFIME_INTERACT_DIV ? col_sd(a.gstats[j * 12 + 6], a.gstats[j * 12 + 7], n)
                                                          : col_sd(cj[0], cj[1], n);
            e1 = kGuardC * sqrt(n) * col_sd(ci[0], ci[1], n) * sd_g;
        }
        double sx, sxx, err;
        if (op == GAFIME_INTERACT_ADD || op == GAFIME_INTERACT_SUB) {
            const double sg = op == GAFIME_INTERACT_ADD ? 1.0 : -1.0;
            sx = ci[0] + sg * cj[0];
            sxx = ci[1] + 2.0 * sg * S1 + cj[1];
            err = kGuardC * (ci[1] + cj[1]) + 2.0 * e1;
        } else {
            sx = S1;
            sxx = S2;
            err = kGuardC * S2 + (2.0 * fabs(S1) * e1 + e1 * e1) / n;
        }
        const double nvar = sxx - sx * sx / n;
        flag = err > kGuardTau * fmax(nvar, 0.0);
    }
    a.flags[((int64_t)oi * a.n_tiles + t) * kTilePairs + e] = flag ? 1 : 0;
    // warp-aggregated append to the re-score list
    const unsigned ballot = __ballot_sync(0xffffffffu, flag);
    if (ballot == 0) return;
    const int lane = threadIdx.x & 31;
    unsigned long long base = 0;
    if (lane == 0) base = atomicAdd(a.count, (unsigned long long)__popc(ballot));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (flag) {
        const unsigned long long slot = base + __popc(ballot & ((1u << lane) - 1u));
        a.list[slot] = make_uint2((uint32_t)t * kTilePairs + (uint32_t)e, (uint32_t)oi);
    }
}

__device__ __forceinline__ float combine(float x, float y, int op, float eps) {
    switch (op) {
        case GAFIME_INTERACT_ADD: return __fadd_rn(x, y);
        case GAFIME_INTERACT_SUB: return __fsub_rn(x, y);
        case GAFIME_INTERACT_DIV: return __fdiv_rn(x, fabsf(y) < eps ? copysignf(eps, y) : y);
        default: return __fmul_rn(x, y);
    }
}

// Persistent CTAs over the flagged (pair, operator) entries: fp64 sums of x, x^2, x*y over
// rows 0 .. n-1 (float4 runs, then the last n % 4 rows one by one), combined in a fixed
// order, then the Pearson of the sums.
__global__ void __launch_bounds__(kRescoreThreads) rescore_kernel(RescoreArgs a) {
    __shared__ double red[kRescoreThreads / 32][3];
    const unsigned long long cnt = *a.count;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t nv = a.n / 4;
    for (unsigned long long q = blockIdx.x; q < cnt; q += gridDim.x) {
        const uint2 ent = a.list[q];
        const int oi = (int)ent.y;
        const int t = (int)(ent.x / kTilePairs), e = (int)(ent.x % kTilePairs);
        const TileCoord tc = a.tiles[t];
        const int64_t i = (int64_t)tc.bi * kTile + e / kTile, j = (int64_t)tc.bj * kTile + e % kTile;
        const int op = a.op[oi];
        const float4* xa = reinterpret_cast<const float4*>(a.x + i * a.ld);
        const float4* xb = reinterpret_cast<const float4*>(a.x + j * a.ld);
        const float4* yv = reinterpret_cast<const float4*>(a.y);
        double s1 = 0.0, s2 = 0.0, s3 = 0.0;
        for (int64_t v = threadIdx.x; v < nv; v += kRescoreThreads) {
            const float4 u = __ldg(xa + v), w = __ldg(xb + v), z = __ldg(yv + v);
            const float xs[4] = {combine(u.x, w.x, op, a.eps), combine(u.y, w.y, op, a.eps),
                                 combine(u.z, w.z, op, a.eps), combine(u.w, w.w, op, a.eps)};
            const float ys[4] = {z.x, z.y, z.z, z.w};
            #pragma unroll
            for (int r = 0; r < 4; ++r) {
                const double xd = (double)xs[r];
                s1 += xd;
                s2 = fma(xd, xd, s2);
                s3 = fma(xd, (double)ys[r], s3);
            }
        }
        if (threadIdx.x < (int)(a.n - 4 * nv)) {
            const int64_t r = 4 * nv + threadIdx.x;
            const double xd = (double)combine(a.x[i * a.ld + r], a.x[j * a.ld + r], op, a.eps);
            s1 += xd;
            s2 = fma(xd, xd, s2);
            s3 = fma(xd, (double)a.y[r], s3);
        }
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
            s3 += __shfl_xor_sync(0xffffffffu, s3, o);
        }
        if (lane == 0) {
            red[warp][0] = s1;
            red[warp][1] = s2;
            red[warp][2] = s3;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double S1 = 0.0, S2 = 0.0, S3 = 0.0;
            for (int w = 0; w < kRescoreThreads / 32; ++w) {
                S1 += red[w][0];
                S2 += red[w][1];
                S3 += red[w][2];
            }
            const double n = a.ystats[0], sum_y = a.ystats[1], var_y = a.ystats[2];
            double r = 0.0;
            if (n > 1.0) {
                const double var_x = S2 - S1 * S1 / n;
                const double cov = S3 - S1 * sum_y / n;
                const double d = var_x * var_y;
                if (d > 0.0) r = cov / sqrt(d);
            }
            a.exact[((int64_t)oi * a.n_tiles + t) * kTilePairs + e] = r;
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_guard(const GuardArgs& g, const RescoreArgs& r, int sm_count, cudaStream_t stream) {
    if (g.n_tiles <= 0) return cudaSuccess;
    if (g.n_ops < 1 || g.n_ops > 4 || (g.gram && !g.gstats)) return cudaErrorInvalidValue;
    if (((uintptr_t)r.x & 15) != 0 || ((uintptr_t)r.y & 15) != 0 || r.ld % 4 != 0 || r.n > r.ld)
        return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(g.count, 0, sizeof(unsigned long long), stream);
    if (e != cudaSuccess) return e;
    guard_kernel<<<dim3((unsigned)g.n_tiles, kTilePairs / kGuardThreads, (unsigned)g.n_ops), kGuardThreads, 0,
                   stream>>>(g);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // a flagged pair costs a full pass over its two columns: enough CTAs to keep every SM
    // streaming; with nothing flagged they return at once
    rescore_kernel<<<(unsigned)(4 * sm_count), kRescoreThreads, 0, stream>>>(r);
    return cudaGetLastError();
}

}  // namespace gafime
