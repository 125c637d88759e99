// CUDA error convention and a small owning device buffer, interface-compatible with the
// reference's include/cuda_support.cuh:1-36 so that code written against the reference
// (its src/main.cu and src/device_matrix.cuh) builds unchanged against this library.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <stdexcept>
#include <vector>

// Throw std::runtime_error carrying the CUDA error string (reference behaviour).
inline void checkCuda(cudaError_t status) {
    if (status != cudaSuccess)
        throw std::runtime_error(cudaGetErrorString(status));
}

// Owns count elements of device memory; a zero count allocates nothing.
template <typename T> class DeviceBuffer {
  public:
    T* ptr = nullptr;

    explicit DeviceBuffer(std::size_t count) {
        if (count != 0)
            checkCuda(cudaMalloc(reinterpret_cast<void**>(&ptr), count * sizeof(T)));
    }
    // Allocate and upload a host vector (synchronous copy).
    explicit DeviceBuffer(const std::vector<T>& host) : DeviceBuffer(host.size()) {
        if (!host.empty())
            checkCuda(cudaMemcpy(ptr, host.data(), host.size() * sizeof(T),
                                 cudaMemcpyHostToDevice));
    }
    ~DeviceBuffer() {
        if (ptr != nullptr)
            cudaFree(ptr);
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};
