// R-MAT workload generated on the GPU (libtcc_workloads; not part of the SpMM operator boundary).
//
// Produces exactly the canonical CSR of tcc_wl_rmat in workloads.cpp: edge e of sampling block
// b = e / 2^22 draws its `scale` quadrant choices from the counter-based stream (seed, b) at
// counters (e - b * 2^22) * scale + level, the (row, column) pairs are sorted and de-duplicated,
// and every entry of row i holds float(1.0 / deg_i) with deg_i the row's distinct columns. One
// thread per edge samples; CUB sorts the keys (row << scale | column, 2 * scale bits) and removes
// duplicates; degrees come from the sorted keys, offsets from an exclusive sum. Scratch: two key
// buffers of 8 bytes per edge sample, the degrees and CUB's temporary storage, freed before the
// call returns.
#include "workloads.h"

#include <cub/cub.cuh>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

void tccWlSetLastError(const char* message);

struct tcc_wl_device_csr {
    uint32_t rows = 0, cols = 0;
    uint64_t nnz = 0;
    uint32_t* rowOffsets = nullptr;
    uint32_t* sourceIds = nullptr;
    float* values = nullptr;
};

namespace {

constexpr uint64_t kSampleBlock = 1ull << 22; // edges per counter stream (as in workloads.cpp)

void check(cudaError_t s) {
    if (s != cudaSuccess)
        throw std::runtime_error(cudaGetErrorString(s));
}

__host__ __device__ inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// Key of counter stream s under seed (the Stream constructor of workloads.cpp).
__host__ __device__ inline uint64_t streamKey(uint64_t seed, uint64_t s) {
    return mix64(seed ^ mix64(s * 0xD6E8FEB86659FD93ull + 1));
}

__global__ void sampleEdges(uint64_t* keys, uint64_t edges, uint32_t scale, uint64_t seed, uint64_t ta, uint64_t tb,
                            uint64_t tc) {
    const uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= edges)
        return;
    const uint64_t block = e / kSampleBlock;
    const uint64_t key = streamKey(seed, block);
    uint64_t counter = (e - block * kSampleBlock) * scale;
    uint32_t r = 0, col = 0;
    for (uint32_t level = 0; level < scale; ++level, ++counter) {
        const uint64_t u = mix64(key + counter * 0x9E3779B97F4A7C15ull);
        const uint32_t bit = 1u << (scale - 1 - level);
        if (u < ta) {
        } else if (u < tb) {
            col |= bit;
        } else if (u < tc) {
            r |= bit;
        } else {
            r |= bit;
            col |= bit;
        }
    }
    keys[e] = (uint64_t(r) << scale) | col;
}

// Degree of every row from the sorted, distinct keys: the entries of row r are the run of keys
// with r in the high bits.
__global__ void countRows(const uint64_t* keys, uint64_t nnz, uint32_t scale, uint32_t* degree) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < nnz)
        atomicAdd(degree + (keys[i] >> scale), 1u);
}

__global__ void fillEntries(const uint64_t* keys, uint64_t nnz, uint32_t scale, const uint32_t* degree,
                            uint32_t* sourceIds, float* values) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nnz)
        return;
    const uint64_t k = keys[i];
    sourceIds[i] = static_cast<uint32_t>(k & ((1ull << scale) - 1));
    values[i] = static_cast<float>(1.0 / static_cast<double>(degree[k >> scale]));
}

template <typename T> T* deviceAlloc(uint64_t count) {
    void* p = nullptr;
    check(cudaMalloc(&p, std::max<uint64_t>(count, 1) * sizeof(T)));
    return static_cast<T*>(p);
}

unsigned blocksFor(uint64_t n) { return static_cast<unsigned>((n + 255) / 256); }

} // namespace

extern "C" {

int tcc_wl_rmat_device(uint32_t scale, uint64_t edges, double a, double b, double c, uint64_t seed, void* stream,
                       tcc_wl_device_csr** out) {
    uint64_t* keyA = nullptr;
    uint64_t* keyB = nullptr;
    uint64_t* selected = nullptr;
    uint32_t* degree = nullptr;
    void* temp = nullptr;
    tcc_wl_device_csr* csr = nullptr;
    try {
        tccWlSetLastError("");
        if (out == nullptr)
            throw std::invalid_argument("null output");
        *out = nullptr;
        if (scale == 0 || scale > 31 || a < 0 || b < 0 || c < 0 || a + b + c > 1.0)
            throw std::invalid_argument("invalid R-MAT parameters");
        if (edges == 0 || edges > 0x7FFFFFFFull)
            throw std::invalid_argument("R-MAT edge samples must be in [1, 2^31)");
        const auto st = static_cast<cudaStream_t>(stream);
        const uint32_t n = 1u << scale;
        // The quadrant thresholds exactly as workloads.cpp computes them (host doubles).
        const uint64_t ta = uint64_t(a * 18446744073709551615.0), tb = uint64_t((a + b) * 18446744073709551615.0),
                       tc = uint64_t((a + b + c) * 18446744073709551615.0);
        keyA = deviceAlloc<uint64_t>(edges);
        keyB = deviceAlloc<uint64_t>(edges);
        selected = deviceAlloc<uint64_t>(1);
        sampleEdges<<<blocksFor(edges), 256, 0, st>>>(keyA, edges, scale, seed, ta, tb, tc);
        check(cudaGetLastError());
        cub::DoubleBuffer<uint64_t> keys(keyA, keyB);
        size_t sortBytes = 0, uniqueBytes = 0, scanBytes = 0;
        check(cub::DeviceRadixSort::SortKeys(nullptr, sortBytes, keys, static_cast<int>(edges), 0, int(2 * scale), st));
        check(cub::DeviceSelect::Unique(nullptr, uniqueBytes, keyA, keyB, selected, static_cast<int>(edges), st));
        check(cub::DeviceScan::ExclusiveSum(nullptr, scanBytes, static_cast<uint32_t*>(nullptr),
                                            static_cast<uint32_t*>(nullptr), static_cast<int>(n) + 1, st));
        size_t tempBytes = std::max(sortBytes, std::max(uniqueBytes, scanBytes));
        check(cudaMalloc(&temp, tempBytes));
        check(cub::DeviceRadixSort::SortKeys(temp, tempBytes, keys, static_cast<int>(edges), 0, int(2 * scale), st));
        uint64_t* sorted = keys.Current();
        uint64_t* unique = keys.Alternate();
        check(cub::DeviceSelect::Unique(temp, tempBytes, sorted, unique, selected, static_cast<int>(edges), st));
        uint64_t nnz = 0;
        check(cudaMemcpyAsync(&nnz, selected, sizeof(uint64_t), cudaMemcpyDeviceToHost, st));
        check(cudaStreamSynchronize(st));
        csr = new tcc_wl_device_csr;
        csr->rows = csr->cols = n;
        csr->nnz = nnz;
        csr->rowOffsets = deviceAlloc<uint32_t>(uint64_t(n) + 1);
        csr->sourceIds = deviceAlloc<uint32_t>(nnz);
        csr->values = deviceAlloc<float>(nnz);
        // Degrees in a zeroed buffer of n + 1 words (the last stays 0), then offsets = exclusive sum.
        degree = deviceAlloc<uint32_t>(uint64_t(n) + 1);
        check(cudaMemsetAsync(degree, 0, (uint64_t(n) + 1) * sizeof(uint32_t), st));
        if (nnz)
            countRows<<<blocksFor(nnz), 256, 0, st>>>(unique, nnz, scale, degree);
        check(cudaGetLastError());
        check(cub::DeviceScan::ExclusiveSum(temp, tempBytes, degree, csr->rowOffsets, static_cast<int>(n) + 1, st));
        if (nnz)
            fillEntries<<<blocksFor(nnz), 256, 0, st>>>(unique, nnz, scale, degree, csr->sourceIds, csr->values);
        check(cudaGetLastError());
        check(cudaStreamSynchronize(st));
        check(cudaFree(temp));
        check(cudaFree(keyA));
        check(cudaFree(keyB));
        check(cudaFree(selected));
        check(cudaFree(degree));
        *out = csr;
        return 0;
    } catch (const std::exception& e) {
        tccWlSetLastError(e.what());
    } catch (...) {
        tccWlSetLastError("unknown error");
    }
    cudaFree(temp);
    cudaFree(keyA);
    cudaFree(keyB);
    cudaFree(selected);
    cudaFree(degree);
    tcc_wl_device_csr_free(csr);
    return 1;
}

int tcc_wl_device_csr_arrays(const tcc_wl_device_csr* csr, uint32_t* rows, uint32_t* cols, uint64_t* nnz,
                             uint32_t** row_offsets, uint32_t** source_ids, float** values) {
    if (csr == nullptr || rows == nullptr || cols == nullptr || nnz == nullptr || row_offsets == nullptr ||
        source_ids == nullptr || values == nullptr) {
        tccWlSetLastError("null argument");
        return 1;
    }
    *rows = csr->rows;
    *cols = csr->cols;
    *nnz = csr->nnz;
    *row_offsets = csr->rowOffsets;
    *source_ids = csr->sourceIds;
    *values = csr->values;
    return 0;
}

void tcc_wl_device_csr_free(tcc_wl_device_csr* csr) {
    if (csr == nullptr)
        return;
    cudaFree(csr->rowOffsets);
    cudaFree(csr->sourceIds);
    cudaFree(csr->values);
    delete csr;
}

} // extern "C"
