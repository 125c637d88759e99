// INT8 feature preparation on sm_100a: per-row absmax quantization, packed16 interleave and
// a one-pass quantize+pack.
//
// Byte parity with the reference (Shixg-cnic/tcc_spmm):
//   quantize: src/format/int8_quantize.cu:4-25  scale = absmax==0 ? 1 : absmax/127.f,
//             q = clamp(lrintf(x/scale), -127, 127), IEEE division, absmax via fmaxf(fabsf)
//   pack16:   src/format/pack_int8.cu:6-15      tile bytes [q0,q8,q1,q9,...,q7,q15]
// The arithmetic per element is the same operation sequence (fmaxf, `/`, lrintf), so the
// bytes agree for every input. The layout differs: the reference runs one 128-thread CTA
// per row and one thread per output u16; here a group of lanes owns a row, every lane owns
// whole 16-feature tiles (four float4 loads, one 16-byte store) and the row maximum is a
// shuffle reduction inside the group. All three kernels are HBM-bound.
#include "common.hpp"

#include <cuda_runtime.h>

namespace tcc {
namespace {

__device__ __forceinline__ int8_t quantizeOne(float x, float scale) {
    const int v = static_cast<int>(lrintf(x / scale));
    return static_cast<int8_t>(v < -127 ? -127 : (v > 127 ? 127 : v));
}

__device__ __forceinline__ unsigned packBytes4(int8_t a, int8_t b, int8_t c, int8_t d) {
    return unsigned(uint8_t(a)) | (unsigned(uint8_t(b)) << 8) | (unsigned(uint8_t(c)) << 16) |
           (unsigned(uint8_t(d)) << 24);
}

// Interleave one 16-byte tile (features 0..15 in w0..w3) into packed16 order.
__device__ __forceinline__ uint4 interleave16(uint4 w) {
    uint4 o;
    o.x = __byte_perm(w.x, w.z, 0x5140); // q0  q8  q1  q9
    o.y = __byte_perm(w.x, w.z, 0x7362); // q2  q10 q3  q11
    o.z = __byte_perm(w.y, w.w, 0x5140); // q4  q12 q5  q13
    o.w = __byte_perm(w.y, w.w, 0x7362); // q6  q14 q7  q15
    return o;
}

// Fast path: features % 16 == 0, x and out 16-byte aligned. A group of GROUP lanes owns a
// row; lane j of the group owns tiles j, j+GROUP, ... (at most TILES of them, kept in
// registers so x is read exactly once). PACKED selects packed16 output order.
template <int GROUP, int TILES, bool PACKED>
__global__ void __launch_bounds__(256) quantizeRowsKernel(const float* __restrict__ x,
                                                          int8_t* __restrict__ out,
                                                          float* __restrict__ scale,
                                                          uint32_t sources, uint32_t features) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t groupLane = lane % GROUP;
    const uint64_t row =
        (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) / GROUP; // one group per row
    const bool active = row < sources;
    const uint32_t tiles = features / 16;
    float4 v[TILES][4];
    float m = 0.0f;
#pragma unroll
    for (int k = 0; k < TILES; ++k) {
        const uint32_t tile = groupLane + k * GROUP;
        if (active && tile < tiles) {
            const float4* src = reinterpret_cast<const float4*>(x + row * features + tile * 16);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                v[k][c] = __ldcs(src + c);
                m = fmaxf(m, fabsf(v[k][c].x));
                m = fmaxf(m, fabsf(v[k][c].y));
                m = fmaxf(m, fabsf(v[k][c].z));
                m = fmaxf(m, fabsf(v[k][c].w));
            }
        }
    }
#pragma unroll
    for (int offset = GROUP / 2; offset > 0; offset >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, offset));
    const float s = m == 0.0f ? 1.0f : m / 127.f;
    if (active && groupLane == 0)
        scale[row] = s;
#pragma unroll
    for (int k = 0; k < TILES; ++k) {
        const uint32_t tile = groupLane + k * GROUP;
        if (active && tile < tiles) {
            uint4 w;
            w.x = packBytes4(quantizeOne(v[k][0].x, s), quantizeOne(v[k][0].y, s),
                             quantizeOne(v[k][0].z, s), quantizeOne(v[k][0].w, s));
            w.y = packBytes4(quantizeOne(v[k][1].x, s), quantizeOne(v[k][1].y, s),
                             quantizeOne(v[k][1].z, s), quantizeOne(v[k][1].w, s));
            w.z = packBytes4(quantizeOne(v[k][2].x, s), quantizeOne(v[k][2].y, s),
                             quantizeOne(v[k][2].z, s), quantizeOne(v[k][2].w, s));
            w.w = packBytes4(quantizeOne(v[k][3].x, s), quantizeOne(v[k][3].y, s),
                             quantizeOne(v[k][3].z, s), quantizeOne(v[k][3].w, s));
            if (PACKED)
                w = interleave16(w);
            *reinterpret_cast<uint4*>(out + row * features + tile * 16) = w;
        }
    }
}

// Any width and alignment: one warp per row, two passes over x.
template <bool PACKED>
__global__ void __launch_bounds__(256) quantizeRowsGeneric(const float* __restrict__ x,
                                                           int8_t* __restrict__ out,
                                                           float* __restrict__ scale,
                                                           uint32_t sources, uint32_t features) {
    const uint32_t lane = threadIdx.x & 31;
    const uint64_t row = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    if (row >= sources)
        return;
    const float* xr = x + row * features;
    float m = 0.0f;
    for (uint32_t j = lane; j < features; j += 32)
        m = fmaxf(m, fabsf(xr[j]));
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, offset));
    const float s = m == 0.0f ? 1.0f : m / 127.f;
    if (lane == 0)
        scale[row] = s;
    int8_t* outRow = out + row * features;
    for (uint32_t j = lane; j < features; j += 32) {
        uint32_t dst = j;
        if (PACKED) { // feature j of tile T lands at byte 2*(j%8) + (j%16 >= 8)
            const uint32_t within = j & 15;
            dst = (j & ~15u) + ((within & 7) << 1) + (within >> 3);
        }
        outRow[dst] = quantizeOne(xr[j], s);
    }
}

// packed16 interleave, one 16-byte tile per thread (q and out 16-byte aligned).
__global__ void __launch_bounds__(256) packTilesKernel(const uint4* __restrict__ q,
                                                       uint4* __restrict__ out, uint64_t tiles) {
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < tiles)
        out[i] = interleave16(__ldcs(q + i));
}

// packed16 interleave for 2-byte aligned buffers: one output u16 per thread.
__global__ void __launch_bounds__(256) packPairsKernel(const int8_t* __restrict__ q,
                                                       unsigned short* __restrict__ out,
                                                       uint64_t pairs) {
    const uint64_t p = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (p < pairs) {
        const uint64_t base = (p >> 3) * 16 + (p & 7);
        out[p] = static_cast<unsigned short>(unsigned(uint8_t(q[base])) |
                                             (unsigned(uint8_t(q[base + 8])) << 8));
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

void checkLaunch() {
    const cudaError_t status = cudaGetLastError();
    if (status != cudaSuccess)
        throw CudaError(cudaGetErrorString(status));
}

template <bool PACKED>
void launchQuantize(const float* x, int8_t* out, float* scale, uint32_t sources, uint32_t features,
                    cudaStream_t stream) {
    // The reference launches an empty grid here, which CUDA rejects (std::runtime_error).
    if (sources == 0 || features == 0)
        throw CudaError("invalid configuration argument");
    if (x == nullptr || out == nullptr || scale == nullptr)
        throw std::invalid_argument("quantize requires non-null buffers");
    if (PACKED && features % 16 != 0)
        throw std::invalid_argument("packed16 requires features % 16 == 0");
    const uint32_t tiles = features / 16;
    const bool fast = features % 16 == 0 && aligned16(x) && aligned16(out) && tiles <= 64;
    constexpr uint32_t block = 256;
    if (fast) {
        // Group size: the smallest power of two >= tiles (max 32); lanes own up to two tiles.
        uint32_t group = 1;
        while (group < tiles && group < 32)
            group <<= 1;
        const uint64_t threads = uint64_t(sources) * group;
        const uint32_t grid = static_cast<uint32_t>((threads + block - 1) / block);
        const bool two = tiles > 32;
        switch (two ? 64 : group) {
#define TCC_Q(G, T)                                                                             \
    quantizeRowsKernel<G, T, PACKED><<<grid, block, 0, stream>>>(x, out, scale, sources, features); \
    break;
        case 1: TCC_Q(1, 1)
        case 2: TCC_Q(2, 1)
        case 4: TCC_Q(4, 1)
        case 8: TCC_Q(8, 1)
        case 16: TCC_Q(16, 1)
        case 32: TCC_Q(32, 1)
        default: TCC_Q(32, 2)
#undef TCC_Q
        }
    } else {
        const uint64_t threads = uint64_t(sources) * 32;
        const uint32_t grid = static_cast<uint32_t>((threads + block - 1) / block);
        quantizeRowsGeneric<PACKED><<<grid, block, 0, stream>>>(x, out, scale, sources, features);
    }
    checkLaunch();
}

} // namespace
} // namespace tcc

extern "C" {

int tcc_quantize_features_int8(const float* x, int8_t* q, float* scale, uint32_t sources,
                               uint32_t features, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchQuantize<false>(x, q, scale, sources, features, reinterpret_cast<cudaStream_t>(stream));
    });
}

int tcc_quantize_pack_features_int8(const float* x, int8_t* packed, float* scale, uint32_t sources,
                                    uint32_t features, tcc_stream_t stream) {
    return tcc::guarded([&] {
        tcc::launchQuantize<true>(x, packed, scale, sources, features,
                                  reinterpret_cast<cudaStream_t>(stream));
    });
}

int tcc_pack_features_int8x16(const int8_t* q, int8_t* packed, uint32_t sources, uint32_t features,
                              tcc_stream_t stream) {
    return tcc::guarded([&] {
        if (sources == 0 || features == 0) // an empty grid in the reference (runtime_error)
            throw tcc::CudaError("invalid configuration argument");
        if (q == nullptr || packed == nullptr)
            throw std::invalid_argument("pack requires non-null buffers");
        if (features % 16 != 0)
            throw std::invalid_argument("packed16 requires features % 16 == 0");
        if ((reinterpret_cast<uintptr_t>(packed) & 1u) != 0)
            throw std::invalid_argument("packed output must be 2-byte aligned");
        const uint64_t bytes = uint64_t(sources) * features;
        const uint64_t lo = reinterpret_cast<uintptr_t>(packed), qlo = reinterpret_cast<uintptr_t>(q);
        if (lo < qlo + bytes && qlo < lo + bytes)
            throw std::invalid_argument("packed output must not alias q");
        auto s = reinterpret_cast<cudaStream_t>(stream);
        constexpr uint32_t block = 256;
        if (tcc::aligned16(q) && tcc::aligned16(packed)) {
            const uint64_t tiles = bytes / 16;
            tcc::packTilesKernel<<<static_cast<uint32_t>((tiles + block - 1) / block), block, 0, s>>>(
                reinterpret_cast<const uint4*>(q), reinterpret_cast<uint4*>(packed), tiles);
        } else {
            const uint64_t pairs = bytes / 2;
            tcc::packPairsKernel<<<static_cast<uint32_t>((pairs + block - 1) / block), block, 0, s>>>(
                q, reinterpret_cast<unsigned short*>(packed), pairs);
        }
        tcc::checkLaunch();
    });
}

} // extern "C"
