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
// The kernels:
//   spmmTmem8Kernel (spmm_tmem8.cuh): the fast path (tcgen05 MMAs, accumulators in tensor
//     memory, 8-panel chunks), used when packedX, Y, the partials, sourceIds, sourceMetadata
//     and values are 16-byte aligned (always true for cudaMalloc'd buffers).
//   spmmPersistentKernel (spmm_persistent.cuh): mma.sync with register accumulators, when
//     only the IDs, metadata or values are not 16-byte aligned.
//   spmmGenericKernel (spmm_generic.cuh): any 2-byte aligned packedX (the reference's own
//     requirement), operands straight from global memory.
// Every wait is bounded (about two seconds of %globaltimer); a wait that runs out records a
// status word (tcc_device_status) and the kernel returns without hanging.
#include "common.hpp"
#include "spmm_generic.cuh"
#include "spmm_persistent.cuh"
#include "spmm_tmem8.cuh"

#include <algorithm>
#include <cuda_runtime.h>
#include <mutex>
#include <string>
#include <vector>

namespace tcc {
namespace {

constexpr int kDefaultVariant = 12; // spmmTmem8Kernel<F, 2>
bool knownVariant(int v) { return v == 0 || v == 1 || v == 2 || v == 3 || v == 12; }

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

// Launch shape of the tensor-memory kernel on `device`. At most Tmem::kMaxCtasPerSm CTAs may
// share an SM's 512 TMEM columns (an allocation beyond them would wait for another CTA to
// finish), so the dynamic shared memory is padded until one more CTA no longer fits. The
// occupancy calculator reports one CTA per SM for kernels that allocate tensor memory, so the
// resident count is derived here from the shared-memory, register and thread limits.
struct LaunchShape {
    uint32_t grid = 0, smem = 0;
    int occupancy = 0; // resident CTAs per SM of this launch shape
};
template <typename L, auto Kernel> LaunchShape tmemShapeOf(int device) {
    static std::mutex mutex;
    static LaunchShape shape[64];
    std::lock_guard<std::mutex> lock(mutex);
    if (device < 0 || device >= 64)
        throw CudaError("device ordinal out of range");
    if (shape[device].grid == 0) {
        int perSmBytes = 0, reserved = 0, optin = 0, sms = 0, regsPerSm = 0, threadsPerSm = 0;
        throwIf(cudaDeviceGetAttribute(&perSmBytes, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device));
        throwIf(cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, device));
        throwIf(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
        throwIf(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        throwIf(cudaDeviceGetAttribute(&regsPerSm, cudaDevAttrMaxRegistersPerMultiprocessor, device));
        throwIf(cudaDeviceGetAttribute(&threadsPerSm, cudaDevAttrMaxThreadsPerMultiProcessor, device));
        const int floor = perSmBytes / (L::kMaxCtasPerSm + 1) - reserved + 1;
        const int bytes = (std::max(L::kBytes, floor) + 127) / 128 * 128;
        if (bytes > optin)
            throw CudaError("tensor-memory SpMM kernel does not fit on this device");
        throwIf(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        cudaFuncAttributes attr{};
        throwIf(cudaFuncGetAttributes(&attr, Kernel));
        // Registers are allocated per warp in units of 256 and each of the 4 SM sub-partitions
        // holds a quarter of the register file; the warps of the resident CTAs spread evenly.
        const int warps = L::kThreads / 32;
        const int regsPerWarp = (attr.numRegs * 32 + 255) / 256 * 256;
        const int warpsPerQuarter = regsPerWarp > 0 ? (regsPerSm / 4) / regsPerWarp : 64;
        int perSm = L::kMaxCtasPerSm;
        perSm = std::min(perSm, perSmBytes / (bytes + reserved));
        perSm = std::min(perSm, threadsPerSm / L::kThreads);
        while (perSm > 0 && (perSm * warps + 3) / 4 > warpsPerQuarter)
            --perSm;
        if (perSm < 1)
            throw CudaError("tensor-memory SpMM kernel does not fit on this device");
        shape[device].occupancy = perSm;
        shape[device].smem = static_cast<uint32_t>(bytes);
        shape[device].grid = static_cast<uint32_t>(perSm * sms);
    }
    return shape[device];
}

template <int F, int P> LaunchShape tmem8Shape(int device) {
    return tmemShapeOf<Tmem8<F, P>, spmmTmem8Kernel<F, P>>(device);
}

template <int F, int P>
void launchTmem8(const tcc_sw32_device_view& m, const int8_t* x, const float* scales, float* y, uint32_t rows,
                 uint32_t cols, float* partials, uint32_t* counters, cudaStream_t stream, uint32_t testFlags) {
    int device = 0;
    throwIf(cudaGetDevice(&device));
    const LaunchShape s = tmem8Shape<F, P>(device);
    const uint32_t grid = std::min<uint32_t>(m.taskCount, s.grid);
    spmmTmem8Kernel<F, P><<<grid, Tmem8<F, P>::kThreads, s.smem, stream>>>(m, x, scales, y, rows, cols, partials,
                                                                           counters, testFlags);
}

// variant: 0 = default fast path (12), 1 = generic kernel, 2/3 = persistent mma.sync kernel with
// 32/64 features per consumer warp, 12 = tensor-memory kernel with 8-panel chunks.
template <int F>
void launch(const tcc_sw32_device_view& m, const int8_t* x, const float* scales, float* y, uint32_t rows,
            uint32_t cols, float* partials, uint32_t* counters, cudaStream_t stream, int variant,
            uint32_t testFlags) {
    const bool fast = aligned(x, 16) && aligned(y, 16) && (partials == nullptr || aligned(partials, 16));
    // Default: the tensor-memory kernel with 8-panel chunks and two producer warps. It moves
    // the IDs, metadata and value ranges with bulk copies, which need 16-byte aligned arrays;
    // otherwise the persistent kernel runs.
    if (variant == 0)
        variant = kDefaultVariant;
    if (variant == 12 && !(aligned(m.sourceIds, 16) && aligned(m.sourceMetadata, 16) && aligned(m.values, 16)))
        variant = F == 128 ? 2 : 3;
    if (variant == 1 || !fast) {
        spmmGenericKernel<F><<<dim3(m.taskCount, F / 128), 128, 0, stream>>>(m, x, scales, y, rows, cols, partials,
                                                                             counters);
    } else if (variant == 2) {
        launchPersistent<F, 32, 1>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else if (variant == 3) {
        launchPersistent<F, 64, 1>(m, x, scales, y, rows, cols, partials, counters, stream);
    } else {
        launchTmem8<F, 2>(m, x, scales, y, rows, cols, partials, counters, stream, testFlags);
    }
    throwIf(cudaGetLastError());
}

void launchChecked(const tcc_sw32_device_view* matrix, const int8_t* packedX, const float* scales, float* output,
                   uint32_t rows, uint32_t cols, uint32_t features, float* partials, uint32_t* counters,
                   cudaStream_t stream, int variant, uint32_t testFlags = 0) {
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
        launch<128>(*matrix, packedX, scales, output, rows, cols, partials, counters, stream, variant, testFlags);
    else
        launch<256>(*matrix, packedX, scales, output, rows, cols, partials, counters, stream, variant, testFlags);
}

// ---- static split-window workspace (tcc_launch_spmm_int8_static_workspace) ---------------
// File-scope device scratch for callers that cannot allocate the partial/counter workspace.
// Zero at module load; every completed launch returns the counters to zero.
constexpr uint64_t kStaticPartialFloats = 2ull << 20; // 8 MiB: partialCount * 8 * features floats
constexpr uint64_t kStaticCounterWords = 1ull << 18;  // 1 MiB: ceil(rows / 32) * features / 128 words
static __device__ __align__(256) float gStaticPartials[kStaticPartialFloats];
static __device__ __align__(256) uint32_t gStaticCounters[kStaticCounterWords];

struct StaticWorkspace {
    float* partials = nullptr;
    uint32_t* counters = nullptr;
};

// Device addresses of the static scratch on the current device, looked up once per device
// (the first call on a device does this setup).
StaticWorkspace staticWorkspace() {
    static std::mutex mutex;
    static StaticWorkspace cache[64];
    int device = 0;
    throwIf(cudaGetDevice(&device));
    if (device < 0 || device >= 64)
        throw CudaError("device ordinal out of range");
    std::lock_guard<std::mutex> lock(mutex);
    StaticWorkspace& w = cache[device];
    if (w.partials == nullptr) {
        void* p = nullptr;
        void* c = nullptr;
        throwIf(cudaGetSymbolAddress(&p, gStaticPartials));
        throwIf(cudaGetSymbolAddress(&c, gStaticCounters));
        w.partials = static_cast<float*>(p);
        w.counters = static_cast<uint32_t*>(c);
    }
    return w;
}

// The launch of tcc_launch_spmm_int8_static_workspace: sizes checked against the static scratch,
// whose device addresses are looked up once per device.
void launchStatic(const tcc_sw32_device_view* matrix, const int8_t* packedX, const float* scales, float* output,
                  uint32_t rows, uint32_t cols, uint32_t features, uint32_t partialCount, cudaStream_t stream,
                  uint32_t testFlags) {
    if (features != 128 && features != 256)
        throw std::invalid_argument("feature dimension must be 128 or 256");
    const uint64_t partialFloats = uint64_t(partialCount) * 8 * features;
    const uint64_t counterWords = partialCount ? (uint64_t(rows) + 31) / 32 * (features / 128) : 0;
    if (partialFloats > kStaticPartialFloats)
        throw std::invalid_argument("split-window partials need " + std::to_string(partialFloats * 4) +
                                    " bytes; the static workspace holds " + std::to_string(kStaticPartialFloats * 4));
    if (counterWords > kStaticCounterWords)
        throw std::invalid_argument("split-window counters need " + std::to_string(counterWords * 4) +
                                    " bytes; the static workspace holds " + std::to_string(kStaticCounterWords * 4));
    const StaticWorkspace w = staticWorkspace();
    launchChecked(matrix, packedX, scales, output, rows, cols, features, partialCount ? w.partials : nullptr,
                  partialCount ? w.counters : nullptr, stream, 0, testFlags);
}

} // namespace
} // namespace tcc

extern "C" {

int tcc_launch_spmm_int8_static_workspace(const tcc_sw32_device_view* matrix, const int8_t* packed_x,
                                          const float* scales, float* output, uint32_t rows, uint32_t cols,
                                          uint32_t features, uint32_t partial_count, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchStatic(matrix, packed_x, scales, output, rows, cols, features, partial_count,
                          reinterpret_cast<cudaStream_t>(stream), 0);
    });
}

int tcc_launch_spmm_int8(const tcc_sw32_device_view* matrix, const int8_t* packed_x, const float* scales,
                         float* output, uint32_t rows, uint32_t cols, uint32_t features, float* partials,
                         uint32_t* counters, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters,
                           reinterpret_cast<cudaStream_t>(stream), 0);
    });
}

// Same contract as tcc_launch_spmm_int8 with an explicit kernel choice (tests and tuning; not
// part of the public header): 0 default (= 12), 1 generic, 2/3 persistent mma.sync (32/64-feature
// consumer warps), 12 tensor-memory with 8-panel chunks.
int tcc_launch_spmm_int8_variant(const tcc_sw32_device_view* matrix, const int8_t* packed_x, const float* scales,
                                 float* output, uint32_t rows, uint32_t cols, uint32_t features, float* partials,
                                 uint32_t* counters, tcc_stream_t stream, int variant) {
    return tcc::guarded([&] {
        if (!tcc::knownVariant(variant))
            throw std::invalid_argument("unknown SpMM kernel variant");
        tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters,
                           reinterpret_cast<cudaStream_t>(stream), variant);
    });
}

// Launch shape of a fast-path kernel variant on the current device (tuning and reports; not
// part of the public header): grid, threads per CTA, dynamic shared memory and the occupancy
// calculator's resident CTAs per SM. Variant 1 (generic) has a per-call grid: reported as 0.
int tcc_spmm_launch_shape(uint32_t features, int variant, uint32_t* grid, uint32_t* threads, uint32_t* smem,
                          int* occupancy) {
    return tcc::guarded([&] {
        if (grid == nullptr || threads == nullptr || smem == nullptr || occupancy == nullptr)
            throw std::invalid_argument("null output");
        if (features != 128 && features != 256)
            throw std::invalid_argument("feature dimension must be 128 or 256");
        if (!tcc::knownVariant(variant))
            throw std::invalid_argument("unknown SpMM kernel variant");
        int device = 0, sms = 1;
        tcc::throwIf(cudaGetDevice(&device));
        tcc::throwIf(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
        if (variant == 0)
            variant = tcc::kDefaultVariant;
        *grid = *threads = *smem = 0;
        *occupancy = 0;
        auto persistent = [&](auto layout, uint32_t g) {
            using L = decltype(layout);
            *grid = g;
            *threads = L::kThreads;
            *smem = L::kBytes;
            *occupancy = static_cast<int>(g) / std::max(1, sms);
        };
        auto tmem = [&](auto layout, tcc::LaunchShape s) {
            using L = decltype(layout);
            *grid = s.grid;
            *threads = L::kThreads;
            *smem = s.smem;
            *occupancy = s.occupancy;
        };
        if (features == 128) {
            switch (variant) {
            case 2: persistent(tcc::Persist<128, 32, 1>{}, tcc::persistentGrid<128, 32, 1>(device)); break;
            case 3: persistent(tcc::Persist<128, 64, 1>{}, tcc::persistentGrid<128, 64, 1>(device)); break;
            case 12: tmem(tcc::Tmem8<128, 2>{}, tcc::tmem8Shape<128, 2>(device)); break;
            default: break;
            }
        } else {
            switch (variant) {
            case 2: persistent(tcc::Persist<256, 32, 1>{}, tcc::persistentGrid<256, 32, 1>(device)); break;
            case 3: persistent(tcc::Persist<256, 64, 1>{}, tcc::persistentGrid<256, 64, 1>(device)); break;
            case 12: tmem(tcc::Tmem8<256, 2>{}, tcc::tmem8Shape<256, 2>(device)); break;
            default: break;
            }
        }
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
        if (s == cudaSuccess && reset) {
            // A launch whose wait ran out skips the tickets of its split windows and leaves their
            // counters short of zero. The caller re-zeroes a workspace it owns; the static
            // workspace's counters are re-zeroed here (the device is idle after the synchronise).
            const tcc::StaticWorkspace w = tcc::staticWorkspace();
            s = cudaMemset(w.counters, 0, tcc::kStaticCounterWords * sizeof(uint32_t));
            if (s == cudaSuccess)
                s = cudaDeviceSynchronize();
        }
        if (s != cudaSuccess)
            throw tcc::CudaError(cudaGetErrorString(s));
    });
}

// ---- failure-path test hooks (not part of the public header) -----------------------------

// tcc_launch_spmm_int8 (static_workspace = 0, caller's partials and counters) or
// tcc_launch_spmm_int8_static_workspace (static_workspace = 1) with the MMA thread of every odd
// CTA of the default kernel stalled on a barrier that nothing completes: its bounded wait runs
// out after about two seconds, the waits of that CTA's other roles run out after it, and status
// bit 0 is set. The split windows whose tasks ran on both even and odd CTAs keep counters short
// of zero. No wait is unbounded and no access leaves the inputs, outputs and workspace.
int tcc_test_launch_spmm_int8_stalled(const tcc_sw32_device_view* matrix, const int8_t* packed_x,
                                      const float* scales, float* output, uint32_t rows, uint32_t cols,
                                      uint32_t features, float* partials, uint32_t* counters, uint32_t partial_count,
                                      int static_workspace, tcc_stream_t stream) {
    return tcc::guarded([&] {
        const auto st = reinterpret_cast<cudaStream_t>(stream);
        if (static_workspace)
            tcc::launchStatic(matrix, packed_x, scales, output, rows, cols, features, partial_count, st,
                              tcc::kTestStallOddCtas);
        else
            tcc::launchChecked(matrix, packed_x, scales, output, rows, cols, features, partials, counters, st, 12,
                               tcc::kTestStallOddCtas);
    });
}

// Number of nonzero words in the static workspace's counters on the current device (synchronises
// the device).
int tcc_test_static_counters_nonzero(uint64_t* nonzero) {
    return tcc::guarded([&] {
        if (nonzero == nullptr)
            throw std::invalid_argument("null output");
        const tcc::StaticWorkspace w = tcc::staticWorkspace();
        std::vector<uint32_t> host(tcc::kStaticCounterWords);
        cudaError_t s = cudaDeviceSynchronize();
        if (s == cudaSuccess)
            s = cudaMemcpy(host.data(), w.counters, host.size() * sizeof(uint32_t), cudaMemcpyDeviceToHost);
        if (s != cudaSuccess)
            throw tcc::CudaError(cudaGetErrorString(s));
        *nonzero = static_cast<uint64_t>(std::count_if(host.begin(), host.end(), [](uint32_t v) { return v != 0; }));
    });
}

} // extern "C"
