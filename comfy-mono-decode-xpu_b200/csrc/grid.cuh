// Grid-wide barrier of a cooperative launch (the role of csrc/mono_common.hpp:54-73 grid_sync), bounded.
//
// counter[0] counts arrivals (epoch * gridDim.x after the epoch-th barrier), counter[1] counts exits; the
// last CTA to exit resets both, so the workspace is reusable by the next launch and by graph replays.
// After kGridSpinLimit polls a waiting CTA records DEV_GRID_TIMEOUT and carries on: no trap, no hang.
#pragma once
#include "common.cuh"

namespace mono {

constexpr uint32_t kGridSpinLimit = 1u << 24;

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Returns false if the wait gave up. flag: one int of shared memory.
__device__ __forceinline__ bool grid_barrier(unsigned* counter, unsigned& epoch, int* flag) {
    __syncthreads();
    ++epoch;
    if (threadIdx.x == 0) {
        const unsigned target = epoch * gridDim.x;
        // one release-add publishes this CTA's writes (ordered by the __syncthreads above); the polls
        // acquire the other CTAs' writes
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
        bool ok = true;
        uint32_t spins = 0;
        const unsigned long long t0 = globaltimer();
        while (ld_acquire_gpu(counter) < target) {
            // short sleeps between polls leave the issue slots to the warps that still stream
            __nanosleep(32);
            if (++spins > kGridSpinLimit || globaltimer() - t0 > kWaitLimitNs) {
                set_device_error(DEV_GRID_TIMEOUT);
                ok = false;
                break;
            }
        }
        *flag = ok;
    }
    __syncthreads();
    return *flag != 0;
}

__device__ __forceinline__ void grid_exit(unsigned* counter) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(counter + 1, 1u) == gridDim.x - 1) {
            atomicExch(counter, 0u);
            atomicExch(counter + 1, 0u);
        }
    }
}

// The same two operations for kernels whose CTA-wide syncs are a named barrier of the first NT threads
// (the consumer warps of a stream kernel; its producer warps never wait at a grid barrier).
template <int BAR, int NT>
__device__ __forceinline__ bool grid_barrier_named(unsigned* counter, unsigned& epoch, int* flag) {
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    ++epoch;
    if (threadIdx.x == 0) {
        const unsigned target = epoch * gridDim.x;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
        bool ok = true;
        uint32_t spins = 0;
        const unsigned long long t0 = globaltimer();
        while (ld_acquire_gpu(counter) < target) {
            if ((++spins & 255) == 0 && globaltimer() - t0 > kWaitLimitNs) {
                set_device_error(DEV_GRID_TIMEOUT);
                ok = false;
                break;
            }
        }
        *flag = ok;
    }
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    return *flag != 0;
}

template <int BAR, int NT>
__device__ __forceinline__ void grid_exit_named(unsigned* counter) {
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(counter + 1, 1u) == gridDim.x - 1) {
            atomicExch(counter, 0u);
            atomicExch(counter + 1, 0u);
        }
    }
}

}  // namespace mono
