// Fused INT8-dequantization SpMM, interface-compatible with the reference's
// include/spmm.cuh:1-23.
#pragma once
#include "format/sw32.h"
#include <cuda_runtime.h>

// Caller-owned scratch of one launch; reusable by launches serialised on one stream.
//   partials: Sw32HostFormat::partialCount * 8 * features floats (no initialisation).
//   counters: ceil(rows/32) * (features/128) u32, zero before the first launch; every
//             launch leaves them zero again.
// Both may be null when partialCount is zero. Concurrent launches need separate
// workspaces, and all buffers must stay alive until the stream has finished.
struct SpmmWorkspace {
    float* partials = nullptr;
    std::uint32_t* counters = nullptr;
};

// Y[rows x features] = A x dequant(packedX) for features 128 or 256
// (std::invalid_argument otherwise). packedX is packed16 INT8 [cols x features], scales
// one float per source, Y row-major FP32; the view must come from the RW-bucketed format
// with its task plan uploaded. Every Y element is overwritten. CUDA launch failures throw
// std::runtime_error; the call itself never synchronises.
void launchSpmmInt8(Sw32DeviceView matrix, const std::int8_t* packedX, const float* scales,
                    float* output, std::uint32_t rows, std::uint32_t cols,
                    std::uint32_t features, SpmmWorkspace workspace,
                    cudaStream_t stream = nullptr);
