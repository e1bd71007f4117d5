// ep.cuh - device helpers of the expert-parallel exchange shared by ep.cu and the down kernels.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace smoe {

// The last of `total` warps to call this: each warp fences its own stores system-wide before it counts, so the
// last one's fence and flag adds order every warp's rows before the flags (the threadfence-reduction pattern).
// Returns true in lane 0 of that warp only; that warp has reset the counter for the next launch.
__device__ __forceinline__ bool ep_last_warp(unsigned* counter, unsigned total) {
    __threadfence_system();
    __syncwarp();
    bool last = false;
    if ((threadIdx.x & 31) == 0) {
        const unsigned prev = atomicAdd(counter, 1u);
        last = prev + 1 == total;
        if (last) {
            __threadfence_system();
            *counter = 0;
        }
    }
    return last;
}

// Called once by every warp that wrote routed rows of a down launch (`total` such warps in the grid).
__device__ __forceinline__ void ep_signal_done(const EpDone& d, unsigned total) {
    if (d.world == 0) return;
    if (ep_last_warp(d.counter, total))
        for (int p = 0; p < d.world; p++) atomicAdd_system(d.flags[p], 1u);
}

// Output row of slot `slot` of a down launch: the plain y unless the launch is expert-parallel.
__device__ __forceinline__ float* down_row(const Work& w, float* y, int slot, int n_out) {
    if (w.slot_pair == nullptr) return y + (size_t) slot * n_out;
    if (slot >= w.shared_base) return w.ep_shared + (size_t) (slot - w.shared_base) * n_out;
    const int p = w.slot_pair[slot];
    const int per = w.ep_rows * w.ep_k;
    return w.ep_out[p / per] + (size_t) (p % per) * n_out;
}

}  // namespace smoe
