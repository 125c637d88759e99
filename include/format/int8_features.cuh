// INT8 feature preparation, interface-compatible with the reference's
// include/format/int8_features.cuh:1-15.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

// X is row-major [sources x features] FP32. Each source row gets its own scale
// absmax/127 (1 for an all-zero row) and q = clamp(round-half-even(x/scale), -127, 127).
// Buffers must be valid, non-aliasing and the sizes nonzero. Launch failures throw
// std::runtime_error; the call only enqueues work on `stream`.
void quantizeFeaturesInt8(const float* x, std::int8_t* q, float* scale, std::uint32_t sources,
                          std::uint32_t features, cudaStream_t stream = nullptr);

// Byte interleave of every 16-feature tile into [q0,q8,q1,q9,...,q7,q15] ("packed16").
// features % 16 == 0; packed holds sources*features bytes, does not alias q and is at
// least 2-byte aligned. Values are not changed.
void packFeaturesInt8x16(const std::int8_t* q, std::int8_t* packed, std::uint32_t sources,
                         std::uint32_t features, cudaStream_t stream = nullptr);
