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
constexpr uint64_t kWaitLimitNs = 2000000000ull; // about two seconds per wait

__device__ __forceinline__ bool boundedWait(uint32_t bar, uint32_t parity) {
    if (dev::mbarTryWait(bar, parity))
        return true;
    const uint64_t start = dev::globalTimerNs();
    for (;;) {
        if (dev::mbarTryWait(bar, parity))
            return true;
        if (dev::globalTimerNs() - start > kWaitLimitNs) {
            atomicOr(&gDeviceStatus, 1u);
            return false;
        }
    }
}
} // namespace
} // namespace tcc
