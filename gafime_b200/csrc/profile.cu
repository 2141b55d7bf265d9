// profile.cu -- per-kernel CUDA-event timing registry.
//
// When enabled (gafime_profile_enable(1)), every kernel launch of the engine is
// bracketed by two CUDA events on the stream it is launched on; gafime_profile_read
// resolves them into total device milliseconds and a launch count per kernel id.
// Disabled (the default) it costs one relaxed atomic load per launch.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "engine.h"

namespace gafime {

namespace {

struct Rec {
    int id;
    int device;
    cudaEvent_t start, stop;
};

std::atomic<int> g_enabled{0};
std::mutex g_mu;
std::vector<Rec> g_recs;

void clear_locked() {
    for (Rec& r : g_recs) {
        cudaEventDestroy(r.start);
        cudaEventDestroy(r.stop);
    }
    g_recs.clear();
}

}  // namespace

KernelTimer::KernelTimer(cudaStream_t stream, int kernel_id) : stream_(stream), id_(kernel_id) {
    if (!g_enabled.load(std::memory_order_relaxed)) return;
    if (cudaEventCreate(&start_) != cudaSuccess) return;
    if (cudaEventCreate(&stop_) != cudaSuccess) {
        cudaEventDestroy(start_);
        return;
    }
    cudaEventRecord(start_, stream_);
    active_ = true;
}

KernelTimer::~KernelTimer() {
    if (!active_) return;
    cudaEventRecord(stop_, stream_);
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_mu);
    g_recs.push_back({id_, dev, start_, stop_});
}

}  // namespace gafime

using namespace gafime;

extern "C" int gafime_profile_enable(int enable) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (enable) clear_locked();  // a new profiling window starts empty; stopping keeps the records
    g_enabled.store(enable ? 1 : 0);
    return GAFIME_SUCCESS;
}

extern "C" int gafime_profile_read(int kernel_id, double* total_ms, int* launches) {
    if (!total_ms || !launches) return GAFIME_ERROR_INVALID_ARGS;
    std::lock_guard<std::mutex> lk(g_mu);
    double ms = 0.0;
    int n = 0;
    int cur = 0;
    cudaGetDevice(&cur);
    for (Rec& r : g_recs) {
        if (kernel_id >= 0 && r.id != kernel_id) continue;
        cudaSetDevice(r.device);
        if (cudaEventSynchronize(r.stop) != cudaSuccess) {
            cudaSetDevice(cur);
            return GAFIME_ERROR_KERNEL_FAILED;
        }
        float e = 0.0f;
        if (cudaEventElapsedTime(&e, r.start, r.stop) != cudaSuccess) {
            cudaSetDevice(cur);
            return GAFIME_ERROR_KERNEL_FAILED;
        }
        ms += e;
        ++n;
    }
    cudaSetDevice(cur);
    *total_ms = ms;
    *launches = n;
    return GAFIME_SUCCESS;
}
