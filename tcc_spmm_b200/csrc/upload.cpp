// Upload of a host SW32 format and its split-task workspace (tcc_device_matrix*), the C-ABI
// counterpart of the reference's DeviceMatrix (src/device_matrix.cuh:8-37): every array copied to
// the current device, partials = partialCount * 8 * features floats and counters = windows *
// (features / 128) u32 set to zero, both only when partialCount > 0. Here all of them share one
// device allocation, each array at a 256-byte aligned offset (the fast kernel's bulk copies need
// 16-byte aligned IDs and metadata).
#include "common.hpp"

#include <cuda_runtime.h>

#include <cstring>

struct tcc_device_matrix {
    void* base = nullptr;
    tcc_sw32_device_view view{};
    float* partials = nullptr;
    uint32_t* counters = nullptr;
};

namespace {

void throwIf(cudaError_t s) {
    if (s != cudaSuccess)
        throw tcc::CudaError(cudaGetErrorString(s));
}

uint64_t alignUp(uint64_t v) { return (v + 255) / 256 * 256; }

} // namespace

extern "C" {

int tcc_device_matrix_upload(const tcc_sw32_sizes* sizes, const tcc_sw32_arrays* arrays, uint32_t features,
                    tcc_stream_t stream, tcc_device_matrix** out) {
    tcc_device_matrix* up = nullptr;
    const int status = tcc::guarded([&] {
        if (sizes == nullptr || arrays == nullptr || out == nullptr)
            throw std::invalid_argument("null argument");
        *out = nullptr;
        if (features != 128 && features != 256)
            throw std::invalid_argument("feature dimension must be 128 or 256");
        if (sizes->windowOffsets == 0)
            throw std::invalid_argument("SW32 format without window offsets");
        const uint64_t windows = sizes->windowOffsets - 1;
        if (sizes->sourceIds != 8 * sizes->rowGroupMasks)
            throw std::invalid_argument("SW32 format: sourceIds must hold 8 entries per panel");
        if (sizes->bucketOffsets != 0 && sizes->bucketOffsets != 17 * windows)
            throw std::invalid_argument("SW32 format: bucketOffsets must hold 17 entries per window");
        if (sizes->tasks > 0xFFFFFFFFull)
            throw std::invalid_argument("SW32 format: more tasks than a view can hold");
        if (sizes->partialCount != 0 && sizes->reductions == 0)
            throw std::invalid_argument("SW32 format: split tasks without reduce ranges");
        struct Piece {
            const void* host;
            uint64_t bytes;
            uint64_t offset;
        };
        Piece pieces[9] = {
            {arrays->windowOffsets, 4 * sizes->windowOffsets, 0},
            {arrays->sourceIds, 4 * sizes->sourceIds, 0},
            {arrays->rowGroupMasks, 4 * sizes->rowGroupMasks, 0},
            {arrays->sourceMetadata, 8 * sizes->sourceIds, 0},
            {arrays->values, 4 * sizes->values, 0},
            {arrays->bucketOffsets, 4 * sizes->bucketOffsets, 0},
            {arrays->tasks, sizeof(tcc_sw32_task) * sizes->tasks, 0},
            {arrays->reductions, sizeof(tcc_sw32_reduce_range) * sizes->reductions, 0},
            {arrays->partialIds, 4 * sizes->partialIds, 0},
        };
        uint64_t total = 0;
        for (Piece& p : pieces) {
            if (p.bytes != 0 && p.host == nullptr)
                throw std::invalid_argument("null host array of a non-empty SW32 array");
            p.offset = total;
            total += alignUp(std::max<uint64_t>(p.bytes, 1));
        }
        const uint64_t partialBytes = sizes->partialCount ? uint64_t(sizes->partialCount) * 8 * features * 4 : 0;
        const uint64_t counterBytes = sizes->partialCount ? windows * (features / 128) * 4 : 0;
        const uint64_t partialOffset = total;
        total += alignUp(partialBytes);
        const uint64_t counterOffset = total;
        total += alignUp(counterBytes);
        up = new tcc_device_matrix;
        throwIf(cudaMalloc(&up->base, total));
        auto* base = static_cast<unsigned char*>(up->base);
        const auto st = reinterpret_cast<cudaStream_t>(stream);
        for (const Piece& p : pieces)
            if (p.bytes)
                throwIf(cudaMemcpyAsync(base + p.offset, p.host, p.bytes, cudaMemcpyHostToDevice, st));
        if (counterBytes)
            throwIf(cudaMemsetAsync(base + counterOffset, 0, counterBytes, st));
        throwIf(cudaStreamSynchronize(st)); // the host arrays may be released after the call
        tcc_sw32_device_view& v = up->view;
        v.windowOffsets = reinterpret_cast<const uint32_t*>(base + pieces[0].offset);
        v.sourceIds = reinterpret_cast<const uint32_t*>(base + pieces[1].offset);
        v.rowGroupMasks = reinterpret_cast<const uint32_t*>(base + pieces[2].offset);
        v.sourceMetadata = reinterpret_cast<const uint64_t*>(base + pieces[3].offset);
        v.values = reinterpret_cast<const float*>(base + pieces[4].offset);
        v.bucketOffsets = reinterpret_cast<const uint32_t*>(base + pieces[5].offset);
        v.tasks = reinterpret_cast<const tcc_sw32_task*>(base + pieces[6].offset);
        v.reductions = reinterpret_cast<const tcc_sw32_reduce_range*>(base + pieces[7].offset);
        v.partialIds = reinterpret_cast<const uint32_t*>(base + pieces[8].offset);
        v.taskCount = static_cast<uint32_t>(sizes->tasks);
        up->partials = partialBytes ? reinterpret_cast<float*>(base + partialOffset) : nullptr;
        up->counters = counterBytes ? reinterpret_cast<uint32_t*>(base + counterOffset) : nullptr;
        *out = up;
    });
    if (status != TCC_OK)
        tcc_device_matrix_free(up);
    return status;
}

int tcc_device_matrix_view(const tcc_device_matrix* upload, tcc_sw32_device_view* view) {
    return tcc::guarded([&] {
        if (upload == nullptr || view == nullptr)
            throw std::invalid_argument("null argument");
        *view = upload->view;
    });
}

int tcc_device_matrix_workspace(const tcc_device_matrix* upload, float** partials, uint32_t** counters) {
    return tcc::guarded([&] {
        if (upload == nullptr || partials == nullptr || counters == nullptr)
            throw std::invalid_argument("null argument");
        *partials = upload->partials;
        *counters = upload->counters;
    });
}

void tcc_device_matrix_free(tcc_device_matrix* upload) {
    if (upload == nullptr)
        return;
    if (upload->base != nullptr)
        cudaFree(upload->base);
    delete upload;
}

} // extern "C"
