// select.cuh -- block-level bitonic sort of top-k candidates (shared by the
// Pearson and mutual-information epilogues).
#pragma once

#include "engine.h"

namespace gafime {

__device__ __forceinline__ void cand_cswap(Cand* s, int i, int j, bool up) {
    // "up": entry i must come before entry j in the final order.
    Cand a = s[i], b = s[j];
    bool sw = up ? cand_before(b, a) : cand_before(a, b);
    if (sw) {
        s[i] = b;
        s[j] = a;
    }
}

// In-place bitonic sort of n (a power of two) shared-memory entries into
// cand_before order.  All threads of the block must call it.
__device__ inline void bitonic_sort(Cand* s, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int e = threadIdx.x; e < n / 2; e += blockDim.x) {
                int i = 2 * stride * (e / stride) + (e % stride);
                cand_cswap(s, i, i + stride, (i & size) == 0);
            }
            __syncthreads();
        }
    }
}

}  // namespace gafime
