// Canonical CSR input, interface-compatible with the reference's include/format/csr.h:1-25.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

// Rows hold strictly increasing source columns with nonzero, finite FP32 weights.
struct CsrMatrix {
    std::vector<std::uint32_t> rowOffsets{0}, sourceIds;
    std::vector<float> values;
};

// A Matrix Market file read into canonical CSR.
struct MtxMatrix {
    std::uint32_t rows, cols;
    CsrMatrix csr;
};

// Read a coordinate real/integer/pattern, general/symmetric Matrix Market file
// (symmetric off-diagonals mirrored, duplicates summed) into canonical CSR.
MtxMatrix loadMatrixMarket(const std::string& path);

// Validate raw CSR arrays, then per row: stable sort by column, sum duplicate columns in
// that order, drop zero sums. Throws std::invalid_argument on bad offsets, columns
// outside [0, cols) or non-finite values.
CsrMatrix makeCanonicalCsr(std::uint32_t rows, std::uint32_t cols, std::uint32_t nnz,
                           const std::uint32_t* rowOffsets, const std::uint32_t* sourceIds,
                           const float* values);
