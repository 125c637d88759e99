// Owner of an uploaded SW32 format and its split-task workspace for C++ callers, the counterpart
// of the reference's DeviceMatrix (src/device_matrix.cuh:8-37), which that library keeps beside
// its CLI rather than in its public headers. Header-only, over the C ABI of libtcc_spmm_b200
// (tcc_device_matrix_*): construct it from a host format and pass view() and workspace() to
// launchSpmmInt8. Errors throw the reference's exception types.
#pragma once

#include "format/sw32.h"
#include "spmm.cuh"
#include "tcc_spmm_b200.h"

#include <cstring>
#include <stdexcept>
#include <string>

namespace tcc {

class DeviceMatrix {
  public:
    // Uploads every array of `matrix` to the current device and allocates the workspace for
    // `features` (128 or 256; counters zeroed), as the reference's constructor does
    // (src/device_matrix.cuh:18-28). The copies are complete when the constructor returns.
    DeviceMatrix(const Sw32HostFormat& matrix, unsigned features, cudaStream_t stream = nullptr) {
        tcc_sw32_sizes sizes{};
        sizes.rows = matrix.rows;
        sizes.cols = matrix.cols;
        sizes.partialCount = matrix.partialCount;
        sizes.bucketed = matrix.bucketOffsets.empty() ? 0u : 1u;
        sizes.windowOffsets = matrix.windowOffsets.size();
        sizes.sourceIds = matrix.sourceIds.size();
        sizes.rowGroupMasks = matrix.rowGroupMasks.size();
        sizes.values = matrix.values.size();
        sizes.bucketOffsets = matrix.bucketOffsets.size();
        sizes.tasks = matrix.tasks.size();
        sizes.reductions = matrix.reductions.size();
        sizes.partialIds = matrix.partialIds.size();
        if (matrix.sourceMetadata.size() != matrix.sourceIds.size())
            throw std::invalid_argument("SW32 format: sourceMetadata and sourceIds differ in size");
        tcc_sw32_arrays arrays{};
        arrays.windowOffsets = matrix.windowOffsets.data();
        arrays.sourceIds = matrix.sourceIds.data();
        arrays.rowGroupMasks = matrix.rowGroupMasks.data();
        arrays.sourceMetadata = matrix.sourceMetadata.data();
        arrays.values = matrix.values.data();
        arrays.bucketOffsets = matrix.bucketOffsets.data();
        arrays.tasks = reinterpret_cast<const tcc_sw32_task*>(matrix.tasks.data());
        arrays.reductions = reinterpret_cast<const tcc_sw32_reduce_range*>(matrix.reductions.data());
        arrays.partialIds = matrix.partialIds.data();
        check(tcc_device_matrix_upload(&sizes, &arrays, features, reinterpret_cast<tcc_stream_t>(stream), &handle_));
    }
    ~DeviceMatrix() { tcc_device_matrix_free(handle_); }
    DeviceMatrix(const DeviceMatrix&) = delete;
    DeviceMatrix& operator=(const DeviceMatrix&) = delete;
    DeviceMatrix(DeviceMatrix&& other) noexcept : handle_(other.handle_) { other.handle_ = nullptr; }
    DeviceMatrix& operator=(DeviceMatrix&& other) noexcept {
        if (this != &other) {
            tcc_device_matrix_free(handle_);
            handle_ = other.handle_;
            other.handle_ = nullptr;
        }
        return *this;
    }

    // The view of all tasks (src/device_matrix.cuh:30-33).
    Sw32DeviceView view() const {
        tcc_sw32_device_view v{};
        check(tcc_device_matrix_view(handle_, &v));
        Sw32DeviceView out;
        static_assert(sizeof(out) == sizeof(v), "Sw32DeviceView ABI");
        std::memcpy(static_cast<void*>(&out), &v, sizeof(out));
        return out;
    }
    // The split-task workspace (src/device_matrix.cuh:35-37); null pointers when partialCount is 0.
    SpmmWorkspace workspace() const {
        SpmmWorkspace w;
        check(tcc_device_matrix_workspace(handle_, &w.partials, &w.counters));
        return w;
    }

  private:
    static void check(int status) {
        if (status == TCC_OK)
            return;
        const std::string message = tcc_last_error();
        if (status == TCC_INVALID_ARGUMENT)
            throw std::invalid_argument(message);
        if (status == TCC_OVERFLOW)
            throw std::overflow_error(message);
        throw std::runtime_error(message);
    }
    tcc_device_matrix* handle_ = nullptr;
};

} // namespace tcc
