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
// finite-input flag) in one file-scope __device__ array of fixed size.
//
// The array costs kScratchBytes (32 MiB) of device memory on every GPU where the
// library is loaded, for the life of the process.  It is shared by all calls, so two
// calls whose work overlaps on the GPU (different streams or threads) race on it; run
// them one after the other.  The first call on each device looks up the array's device
// address with cudaGetSymbolAddress (see device_scratch below); make that first call
// before any stream capture begins.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "engine.h"

namespace gafime {

namespace {

constexpr int kMaxFeatures = GAFIME_NOALLOC_MAX_FEATURES;       // 256 -> at most 10 pair tiles
constexpr int64_t kMaxRows = GAFIME_NOALLOC_MAX_ROWS;           // 2,097,152 padded rows
constexpr int kMaxTileSplits = 170;                              // tiles x row splits
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
constexpr size_t kScratchBytes = 32u << 20;
static_assert(kFlagOff + 256 <= kScratchBytes, "no-alloc scratch layout exceeds its array");

// The scratch itself.  Host code must not use this name as a pointer: on the host it
// only stands for the symbol; device_scratch() returns its real device address.
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device
// (with that device current) and cached.
cudaError_t device_scratch(unsigned char** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_addr[dev] = static_cast<unsigned char*>(p);
    }
    *out = g_addr[dev];
    return cudaSuccess;
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

    int dev = 0, sm = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);

    // finite inputs only, as gafime_allpairs_scores (the flag must start at zero)
    e = cudaMemsetAsync(flag, 0, sizeof(int), s);
    if (e != cudaSuccess) return status_from(e);
    finite_kernel<<<4 * sm, 256, 0, s>>>(d_x, f, ld, n, flag);
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
    e = launch_epilogue_topk(a, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return status_from(e);
}
