// C++ drop-in device entry points with the reference signatures (include/spmm.cuh,
// include/format/int8_features.cuh). Each forwards to the C ABI and turns a nonzero status
// into the exception the reference throws: std::invalid_argument for a bad feature count
// (reference src/kernel/spmm.cu:28), std::runtime_error for CUDA failures (reference
// include/cuda_support.cuh:8-11).
#include "common.hpp"
#include "format/int8_features.cuh"
#include "spmm.cuh"

#include <cstring>

void launchSpmmInt8(Sw32DeviceView matrix, const std::int8_t* packedX, const float* scales, float* output,
                    std::uint32_t rows, std::uint32_t cols, std::uint32_t features, SpmmWorkspace workspace,
                    cudaStream_t stream) {
    tcc_sw32_device_view view;
    static_assert(sizeof(view) == sizeof(matrix), "Sw32DeviceView ABI");
    std::memcpy(&view, &matrix, sizeof(view));
    tcc::check(tcc_launch_spmm_int8(&view, packedX, scales, output, rows, cols, features, workspace.partials,
                                    workspace.counters, reinterpret_cast<tcc_stream_t>(stream)));
}

void quantizeFeaturesInt8(const float* x, std::int8_t* q, float* scale, std::uint32_t sources,
                          std::uint32_t features, cudaStream_t stream) {
    tcc::check(tcc_quantize_features_int8(x, q, scale, sources, features, reinterpret_cast<tcc_stream_t>(stream)));
}

void packFeaturesInt8x16(const std::int8_t* q, std::int8_t* packed, std::uint32_t sources, std::uint32_t features,
                         cudaStream_t stream) {
    tcc::check(tcc_pack_features_int8x16(q, packed, sources, features, reinterpret_cast<tcc_stream_t>(stream)));
}
