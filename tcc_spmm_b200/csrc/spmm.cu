// Fused Y = A x dequant(X_int8) SpMM over the SW32 panel format, sm_100a: launcher and C ABI.
//
// Replaces the reference kernel spmmInt8Kernel<F> and its launcher (Shixg-cnic/tcc_spmm
// src/kernel/spmm_kernel.cuh:172-283, src/kernel/spmm.cu:1-31) behind the same arrays and
// workspace contract. Kept from the reference because the ABI or the numbers depend on it: the
// SW32 panel/task/partial layouts, TF32 operands rounded to nearest with ties away from zero,
// FP32 accumulation on tensor cores, the direct write of unsplit tasks, the partial blocks
// [partialCount][8][F] of split tasks and the last-arriver merge with a wrapping
// acquire-release ticket that returns every counter to zero.
//
// Two kernels:
//   spmmPersistentKernel (spmm_persistent.cuh): the fast path, used when packedX, Y and the
//     partials are 16-byte aligned (always true for cudaMalloc'd buffers).
//   spmmGenericKernel (spmm_generic.cuh): any 2-byte aligned packedX (the reference's own
//     requirement), operands straight from global memory.
// Every wait is bounded (about two seconds of %globaltimer); a wait that runs out records a
// status word (tcc_device_status) and the kernel returns without hanging.
#include "common.hpp"
#include "spmm_generic.cuh"
#include "spmm_persistent.cuh"

#include <cuda_runtime.h>
#include <mutex>

namespace tcc {
namespace {

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

void throwIf(cudaError_t s) {
    if (s != cudaSuccess)
        throw CudaError(cudaGetErrorString(s));
}

// Grid of the persistent kernel on `device`: SMs x resident CTAs per SM (computed once per
// device and kernel variant).
template <int F, int FPW, int P> uint32_t persistentGrid(int device) {
    static std::mutex mutex;
    static int grid[64] = {};
    std::lock_guard<std::mutex> lock(mutex);
    if (device < 0 || device >= 64)
        throw CudaError("device ordinal out of range");
    if (grid[device] == 0) {
        using L = Persist<F, FPW, P>;
        throwIf(cudaFuncSetAttribute(spmmPersistentKernel<F, FPW, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     L::kBytes));
        int perSm = 0, sms = 0;
        throwIf(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&perSm, spmmPersistentKernel<F, FPW, P>, L::kThreads,
                                                              L::kBytes));
        throwIf(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        if (perSm < 1)
            throw CudaError("persistent SpMM kernel does not fit on this device");
        grid[device] = perSm * sms;
    }
    return static_cast<uint32_t>(grid[device]);
}

template <int F, int FPW, int P>
void launchPersistent(const tcc_sw32_device_view& m, const int8_t* x, const float* scales, float* y, uint32_t rows,
                      uint32_t cols, float* partials, uint32_t* counters, cudaStream_t stream) {
    int device = 0;
    throwIf(cudaGetDevice(&device));
    const uint32_t grid = std::min<uint32_t>(m.taskCount, persistentGrid<F, FPW, P>(device));
    spmmPersistentKernel<F, FPW, P><<<grid, Persist<F, FPW, P>::kThreads, Persist<F, FPW, P>::kBytes, stream>>>(
        m, x, scales, y, rows, cols, partials, counters);
}

// variant: 0 = default fast path, 1 = generic kernel, 2/3 = persistent kernel with 32/64
// features per consumer warp and one producer warp, 4/5 = the same with two producer warps,
// 6/7 = with four producer warps.
template <int F>
void launch(const tcc_sw32_device_view& m, const int8_t* x, const float* scales, float* y, uint32_t rows,
            uint32_t cols, float* partials, uint32_t* counters, cudaStream_t stream, int variant) {
    const bool fast = aligned(x, 16) && aligned(y, 16) && (partials == nullptr || aligned(partials, 16));
    if (variant == 0)
        variant = F == 128 ? 2 : 3;
    if (variant == 1 || !fast) {
        spmmGenericKernel<F><<<dim3(m.taskCount, F / 128), 128, 0, stream>>>(m, x, scales, y, rows, cols, partials,
                                                                             counters);
    } else if (variant == 2) {
        launchPersistent<F, 32, 1>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else if (variant == 3) {
        launchPersistent<F, 64, 1>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else if (variant == 4) {
        launchPersistent<F, 32, 2>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else if (variant == 5) {
        launchPersistent<F, 64, 2>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else if (variant == 6) {
        launchPersistent<F, 32, 4>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else {
        launchPersistent<F, 64, 4>(m, x, scales, y, rows, cols, partials, counters, stream);
    }
    throwIf(cudaGetLastError());
}

void launchChecked(const tcc_sw32_device_view* matrix, const int8_t* packedX, const float* scales, float* output,
                   uint32_t rows, uint32_t cols, uint32_t features, float* partials, uint32_t* counters,
                   cudaStream_t stream, int variant) {
    if (matrix == nullptr)
        throw std::invalid_argument("null SW32 device view");
    if (features != 128 && features != 256)
        throw std::invalid_argument("feature dimension must be 128 or 256");
    if (matrix->taskCount == 0) // the reference launches an empty grid (std::runtime_error)
        throw CudaError("invalid configuration argument");
    if (matrix->tasks == nullptr || matrix->sourceIds == nullptr || matrix->sourceMetadata == nullptr ||
        matrix->rowGroupMasks == nullptr || packedX == nullptr || scales == nullptr || output == nullptr)
        throw std::invalid_argument("null device array in launchSpmmInt8");
    if (!aligned(packedX, 2) || !aligned(output, 4))
        throw std::invalid_argument("packedX must be 2-byte and Y 4-byte aligned");
    if (features == 128)
        launch<128>(*matrix, packedX, scales, output, rows, cols, partials, counters, stream, variant);
    else
        launch<256>(*matrix, packedX, scales, output, rows, cols, partials, counters, stream, variant);
}

} // namespace
} // namespace tcc

extern "C" {

int tcc_launch_spmm_int8(const tcc_sw32_device_view* matrix, const int8_t* packed_x, const float* scales,
                         float* output, uint32_t rows, uint32_t cols, uint32_t features, float* partials,
                         uint32_t* counters, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters,
                           reinterpret_cast<cudaStream_t>(stream), 0);
    });
}

// Same contract as tcc_launch_spmm_int8 with an explicit kernel choice (tests and tuning; not
// part of the public header): 0 default, 1 generic, 2/3 persistent with 32/64-feature
// consumer warps.
int tcc_launch_spmm_int8_variant(const tcc_sw32_device_view* matrix, const int8_t* packed_x, const float* scales,
                                 float* output, uint32_t rows, uint32_t cols, uint32_t features, float* partials,
                                 uint32_t* counters, tcc_stream_t stream, int variant) {
    return tcc::guarded([&] {
        if (variant < 0 || variant > 7)
            throw std::invalid_argument("unknown SpMM kernel variant");
        tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters,
                           reinterpret_cast<cudaStream_t>(stream), variant);
    });
}

int tcc_device_status(uint32_t* status, int reset) {
    return tcc::guarded([&] {
        if (status == nullptr)
            throw std::invalid_argument("null status");
        cudaError_t s = cudaDeviceSynchronize();
        if (s == cudaSuccess)
            s = cudaMemcpyFromSymbol(status, tcc::gDeviceStatus, sizeof(uint32_t));
        if (s == cudaSuccess && reset) {
            const uint32_t zero = 0;
            s = cudaMemcpyToSymbol(tcc::gDeviceStatus, &zero, sizeof(uint32_t));
        }
        if (s != cudaSuccess)
            throw tcc::CudaError(cudaGetErrorString(s));
    });
}

} // extern "C"
