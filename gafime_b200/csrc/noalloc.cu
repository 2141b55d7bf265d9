// noalloc.cu -- all-pairs Pearson scores for callers that cannot allocate GPU memory.
//
// Who needs this: a host program that already owns the whole device-memory budget
// (an arena or caching allocator that reserves most of the GPU up front, a database or
// serving process that hands this library device buffers it carved out itself) cannot
// let a library call cudaMalloc behind its back -- the call can fail for lack of room,
// fragment the owner's pool, or stall other streams with the implicit device-wide
// synchronisation that cudaMalloc/cudaFree may perform.  Such a caller passes its own
// device input and output buffers, and this entry point keeps every intermediate
// (column statistics, the centred target, per-tile moment partials, the tile list, the
// finite-input flag, the accuracy guard's flags, re-score list and exact scores, a copy of
// the target) in one file-scope __device__ array of fixed size.  The moments come from the
// CUDA-core pair-moment kernel (fp32 products in runs of 256 rows, fp64 across runs); the
// pairs it cannot hold to 1e-4 are re-scored exactly, as in gafime_allpairs_scores.
//
// The array costs kScratchBytes (32 MiB) of device memory on every GPU where the
// library is loaded, for the life of the process.  It is shared by all calls, so two
// calls whose work overlaps on the GPU (different streams or threads) race on it; run
// them one after the other.  The first call on each device (and the first after that
// device's context was re-created, e.g. by cudaDeviceReset) looks up the array's device
// address with cudaGetSymbolAddress (see device_scratch below); make that first call
// before any stream capture begins.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "engine.h"

namespace gafime {

namespace {

constexpr int kMaxFeatures = GAFIME_NOALLOC_MAX_FEATURES;       // 256 -> at most 10 pair tiles
constexpr int64_t kMaxRows = GAFIME_NOALLOC_MAX_ROWS;           // 2,097,152 padded rows
constexpr int kMaxTileSplits = 150;                              // tiles x row splits
constexpr int kMaxTiles = 10;                                    // 64-tiles of 256 features
constexpr int kMaxColSplits = 2048;                              // (column, split) partials

// Scratch layout (byte offsets, each 256-aligned).
constexpr size_t kMomentsOff = 0;
constexpr size_t kMomentsBytes = (size_t)kMaxTileSplits * 3 * kTilePairs * sizeof(double);
constexpr size_t kYcenOff = (kMomentsOff + kMomentsBytes + 255) / 256 * 256;
constexpr size_t kYcenBytes = (size_t)kMaxRows * sizeof(float);
constexpr size_t kStatsOff = (kYcenOff + kYcenBytes + 255) / 256 * 256;
constexpr size_t kStatsBytes = (size_t)(kMaxFeatures * 4 + 8) * sizeof(double);
constexpr size_t kPartOff = (kStatsOff + kStatsBytes + 255) / 256 * 256;
constexpr size_t kPartBytes = (size_t)kMaxColSplits * 3 * sizeof(double);
constexpr size_t kTilesOff = (kPartOff + kPartBytes + 255) / 256 * 256;
constexpr size_t kTilesBytes = 64 * sizeof(TileCoord);
constexpr size_t kFlagOff = (kTilesOff + kTilesBytes + 255) / 256 * 256;
constexpr size_t kYOff = kFlagOff + 256;                         // copy of the target (16-byte aligned)
constexpr size_t kYBytes = (size_t)kMaxRows * sizeof(float);
constexpr size_t kGuardCountOff = (kYOff + kYBytes + 255) / 256 * 256;
constexpr size_t kGuardFlagsOff = kGuardCountOff + 256;
constexpr size_t kGuardFlagsBytes = (size_t)kMaxTiles * kTilePairs;
constexpr size_t kGuardExactOff = (kGuardFlagsOff + kGuardFlagsBytes + 255) / 256 * 256;
constexpr size_t kGuardExactBytes = (size_t)kMaxTiles * kTilePairs * sizeof(double);
constexpr size_t kGuardListOff = (kGuardExactOff + kGuardExactBytes + 255) / 256 * 256;
constexpr size_t kGuardListBytes = (size_t)kMaxTiles * kTilePairs * sizeof(uint2);
constexpr size_t kScratchEnd = kGuardListOff + kGuardListBytes;
constexpr size_t kScratchBytes = 32u << 20;
static_assert(kScratchEnd <= kScratchBytes, "no-alloc scratch layout exceeds its array");
static_assert((kMaxFeatures + kTile - 1) / kTile * ((kMaxFeatures + kTile - 1) / kTile + 1) / 2 <= kMaxTiles,
              "guard regions hold every tile");

// The scratch itself.  Host code must not use this name as a pointer: on the host it
// only stands for the symbol; device_scratch() returns its real device address.
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {};
CUcontext g_ctx[kMaxDevices] = {};

// The driver's current context (the device's primary context under the runtime), read
// through the runtime's driver entry point so the library needs no libcuda link.
CUcontext current_context() {
    using GetCurrent = CUresult (*)(CUcontext*);
    static GetCurrent fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetCurrent>(p);
    });
    CUcontext c = nullptr;
    if (fn) fn(&c);
    return c;
}

// Device address of g_noalloc_scratch on the current device, looked up once per device
// (with that device current) and cached.  The cache is keyed on the device's context as
// well: cudaDeviceReset ends the context, and the new one loads the module again at a new
// address, which the next call then looks up.
cudaError_t device_scratch(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    // a thread the runtime has not bound to the context yet reads none: look up again
    const CUcontext ctx = current_context();
    if (!g_addr[dev] || !ctx || g_ctx[dev] != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // initialises the context if needed
        if (e != cudaSuccess) return e;
        g_addr[dev] = static_cast<unsigned char*>(p);
        g_ctx[dev] = current_context();
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

// Input check over the caller's matrix: rows below n must be finite, rows n .. ld-1 must be
// zero (the moment kernel sums every row of a column).  flag |= 1 otherwise.
__global__ void noalloc_input_check_kernel(const float* __restrict__ x, int64_t cols, int64_t ld, int64_t n,
                                           int* __restrict__ flag) {
    const int64_t total = cols * ld;
    int bad = 0;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[e];
        bad |= (e % ld < n) ? !isfinite(v) : (v != 0.0f);
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1);
}

// Upper-triangle 64 x 64 tiles in row-major order (one thread; at most 10 tiles).
__global__ void noalloc_tiles_kernel(int nb, TileCoord* tiles) {
    int t = 0;
    for (int bi = 0; bi < nb; ++bi)
        for (int bj = bi; bj < nb; ++bj) tiles[t++] = TileCoord{bi, bj};
}

int col_splits(int64_t cols, int64_t n, int sm) {
    int64_t want = (4 * (int64_t)sm + cols - 1) / cols;
    want = std::min<int64_t>(want, (n + 4095) / 4096);
    want = std::min<int64_t>(want, kMaxColSplits / cols);
    return (int)std::max<int64_t>(1, want);
}

}  // namespace

}  // namespace gafime

using namespace gafime;

extern "C" int gafime_allpairs_scores_noalloc(const float* d_x, int64_t ld, const float* d_y,
                                              int n_samples, int n_features, int interact_type,
                                              float div_eps, double* d_scores_out, void* stream) {
    if (!d_x || !d_y || !d_scores_out) return GAFIME_ERROR_INVALID_ARGS;
    if (n_samples < 1 || n_features < 1 || n_features > kMaxFeatures) return GAFIME_ERROR_INVALID_ARGS;
    if (ld < n_samples || ld % kRowPad != 0 || ld > kMaxRows) return GAFIME_ERROR_INVALID_ARGS;
    if (((uintptr_t)d_x & 15) != 0) return GAFIME_ERROR_INVALID_ARGS;
    if (interact_type < GAFIME_INTERACT_MULT || interact_type > GAFIME_INTERACT_DIV) return GAFIME_ERROR_INVALID_ARGS;
    if (!(div_eps > 0.0f)) return GAFIME_ERROR_INVALID_ARGS;
    const int64_t f = n_features, n = n_samples;
    if (f < 2) return GAFIME_SUCCESS;  // no pairs
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    unsigned char* base = nullptr;
    cudaError_t e = device_scratch(&base);
    if (e != cudaSuccess) return status_from(e);
    double* moments = reinterpret_cast<double*>(base + kMomentsOff);
    float* ycen = reinterpret_cast<float*>(base + kYcenOff);
    double* colstats = reinterpret_cast<double*>(base + kStatsOff);
    double* ycol = colstats + f * 4;
    double* ystats = ycol + 4;
    double* part = reinterpret_cast<double*>(base + kPartOff);
    TileCoord* tiles = reinterpret_cast<TileCoord*>(base + kTilesOff);
    int* flag = reinterpret_cast<int*>(base + kFlagOff);
    float* y_copy = reinterpret_cast<float*>(base + kYOff);

    int dev = 0, sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);

    // finite inputs only, as gafime_allpairs_scores, and zero padding rows (the flag must
    // start at zero)
    e = cudaMemsetAsync(flag, 0, sizeof(int), s);
    if (e != cudaSuccess) return status_from(e);
    noalloc_input_check_kernel<<<4 * sm, 256, 0, s>>>(d_x, f, ld, n, flag);
    finite_kernel<<<4 * sm, 256, 0, s>>>(d_y, 1, n, n, flag);
    int h_flag = 0;
    e = cudaMemcpyAsync(&h_flag, flag, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return status_from(e);
    if (h_flag) return GAFIME_ERROR_INVALID_ARGS;

    // target statistics and the centred target (zero beyond n, up to ld)
    int ys = col_splits(1, n, sm);
    int64_t yspan = ((n + ys - 1) / ys + 255) / 256 * 256;
    col_partial_kernel<<<dim3(1, ys), 256, 0, s>>>(d_y, n, n, nullptr, yspan, part);
    col_combine_kernel<<<1, 128, 0, s>>>(part, 1, ys, n, ycol);
    ystats_kernel<<<1, 1, 0, s>>>(ycol, n, ystats);
    ycen_kernel<<<4 * sm, 256, 0, s>>>(d_y, n, ld, ystats, ycen);
    // column sums: sum x, sum x^2, sum x*ycen
    int xs = col_splits(f, n, sm);
    int64_t xspan = ((n + xs - 1) / xs + 255) / 256 * 256;
    col_partial_kernel<<<dim3((unsigned)f, xs), 256, 0, s>>>(d_x, ld, n, ycen, xspan, part);
    col_combine_kernel<<<(unsigned)((f + 127) / 128), 128, 0, s>>>(part, (int)f, xs, n, colstats);

    // pair tiles and row splits (tiles x splits bounded by the moment region)
    const int nb = (int)((f + kTile - 1) / kTile);
    const int nt = nb * (nb + 1) / 2;
    noalloc_tiles_kernel<<<1, 1, 0, s>>>(nb, tiles);
    int splits = std::max(1, std::min(sm / nt, kMaxTileSplits / nt));
    splits = (int)std::min<int64_t>(splits, std::max<int64_t>(1, ld / 1024));
    int64_t rps = ((ld + splits - 1) / splits + kRowPad - 1) / kRowPad * kRowPad;
    splits = (int)((ld + rps - 1) / rps);
    e = cudaGetLastError();
    if (e != cudaSuccess) return status_from(e);

    e = launch_pair_moments(d_x, ld, ycen, f, tiles, nt, splits, rps,
                            interact_type == GAFIME_INTERACT_DIV, div_eps, moments, s);
    if (e != cudaSuccess) return status_from(e);
    EpilogueArgs a;
    memset(&a, 0, sizeof(a));
    a.moments[0] = moments;
    a.splits[0] = splits;
    a.op[0] = interact_type;
    a.cands[0] = nullptr;  // scores only
    a.n_ops = 1;
    a.tiles = tiles;
    a.n_tiles = nt;
    a.f = f;
    a.colstats = colstats;
    a.ystats = ystats;
    a.k_pad = 1;
    a.sub_lists = 1;
    a.all_scores = d_scores_out;
    {
        // accuracy guard and exact re-score, as the allocating entry points run them (the
        // re-score reads the target from a 16-byte aligned copy in the scratch array)
        GuardArgs g;
        memset(&g, 0, sizeof(g));
        RescoreArgs r;
        memset(&r, 0, sizeof(r));
        g.moments[0] = moments;
        g.splits[0] = splits;
        g.op[0] = r.op[0] = interact_type;
        g.n_ops = 1;
        g.tiles = r.tiles = tiles;
        g.n_tiles = r.n_tiles = nt;
        g.f = f;
        g.colstats = colstats;
        g.ystats = r.ystats = ystats;
        g.gram = 0;
        g.flags = reinterpret_cast<uint8_t*>(base + kGuardFlagsOff);
        g.count = reinterpret_cast<unsigned long long*>(base + kGuardCountOff);
        g.list = reinterpret_cast<uint2*>(base + kGuardListOff);
        r.x = d_x;
        r.y = y_copy;
        r.ld = ld;
        r.n = n;
        r.eps = div_eps;
        r.count = g.count;
        r.list = g.list;
        r.exact = reinterpret_cast<double*>(base + kGuardExactOff);
        e = cudaMemcpyAsync(y_copy, d_y, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) e = launch_guard(g, r, sm, s);
        if (e != cudaSuccess) return status_from(e);
        a.guard_flags = g.flags;
        a.exact = r.exact;
    }
    e = launch_epilogue_topk(a, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return status_from(e);
}
