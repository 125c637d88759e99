// Definitions shared by the SpMM kernels.
#pragma once
#include "common.hpp"
#include "spmm_device.cuh"

namespace tcc {

// Status word of bounded device waits and workspace misuse (read by tcc_device_status):
//   bit 0: an mbarrier wait ran out; bit 1: a split task found no partial/counter workspace.
// Defined here: the SpMM kernels and their launcher form one translation unit (spmm.cu).
__device__ unsigned int gDeviceStatus = 0;

namespace {
constexpr uint32_t kNoPartial = 0xFFFFFFFFu;
// Window index of a padding entry in a task order built for a persistent grid
// (tcc_balance_tasks_padded): it has no panels and no rows, and every kernel skips it.
constexpr uint32_t kSkipTask = 0xFFFFFFFFu;
constexpr uint64_t kWaitLimitNs = 2000000000ull; // about two seconds per wait

// Wait for the given phase of an mbarrier. The warp is suspended by the hardware between
// attempts (no busy spin); the timer is read once every 64 attempts and the wait gives up
// after kWaitLimitNs, recording bit 0 of the status word.
__device__ __forceinline__ bool boundedWait(uint32_t bar, uint32_t parity) {
    if (dev::mbarTryWait(bar, parity))
        return true;
    uint64_t start = 0;
    for (uint32_t attempt = 1;; ++attempt) {
        if (dev::mbarTryWaitSuspend(bar, parity, 2000u))
            return true;
        if ((attempt & 63u) == 0) {
            const uint64_t now = dev::globalTimerNs();
            if (start == 0) {
                start = now;
            } else if (now - start > kWaitLimitNs) {
                atomicOr(&gDeviceStatus, 1u);
                return false;
            }
        }
    }
}
// Bounded wait for waits that are usually long (a warp that waits on another role's
// progress): between attempts the warp sleeps 32 ns, doubling to 256 ns, instead of retrying
// at once, so it takes almost no issue slots from the warps doing the work.
__device__ __forceinline__ bool boundedWaitBackoff(uint32_t bar, uint32_t parity) {
    if (dev::mbarTryWait(bar, parity))
        return true;
    const uint64_t start = dev::globalTimerNs();
    uint32_t ns = 32;
    for (;;) {
        __nanosleep(ns);
        if (dev::mbarTryWait(bar, parity))
            return true;
        ns = ns < 256u ? 2 * ns : 256u;
        if (dev::globalTimerNs() - start > kWaitLimitNs) {
            atomicOr(&gDeviceStatus, 1u);
            return false;
        }
    }
}
} // namespace
} // namespace tcc
