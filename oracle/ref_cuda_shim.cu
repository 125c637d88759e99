// ORACLE - test infrastructure, not product code.
// extern "C" wrapper around the reference's own CUDA entry points (Shixg-cnic/tcc_spmm
// src/kernel/spmm.cu, src/format/int8_quantize.cu, src/format/pack_int8.cu), compiled from
// the reference sources into oracle/_ref by oracle/build.py: once as compute_80 PTX (the
// reference's default architecture, JIT-compiled by the driver on the B200) and once for
// sm_100a. Used by GPU tests as a second oracle for q, scales, packed bytes and Y, and by
// bench.py --impl reference to time the reference kernel beside the CPU baseline.
#include "format/int8_features.cuh"
#include "spmm.cuh"

#include <cstring>
#include <stdexcept>

#define EXPORT extern "C" __attribute__((visibility("default")))

namespace {
template <typename Body> int call(char* err, int errlen, Body&& body) {
    try {
        body();
        return 0;
    } catch (const std::exception& e) {
        if (err && errlen > 0) {
            std::strncpy(err, e.what(), errlen - 1);
            err[errlen - 1] = '\0';
        }
        return dynamic_cast<const std::invalid_argument*>(&e) ? 1 : 3;
    }
}
} // namespace

// view: the nine pointers and task count laid out as Sw32DeviceView.
EXPORT int ref_launch_spmm_int8(const void* view, const std::int8_t* packedX, const float* scales, float* output,
                                std::uint32_t rows, std::uint32_t cols, std::uint32_t features, float* partials,
                                std::uint32_t* counters, void* stream, char* err, int errlen) {
    return call(err, errlen, [&] {
        Sw32DeviceView v;
        std::memcpy(&v, view, sizeof(v));
        launchSpmmInt8(v, packedX, scales, output, rows, cols, features, SpmmWorkspace{partials, counters},
                       static_cast<cudaStream_t>(stream));
    });
}

EXPORT int ref_quantize_features_int8(const float* x, std::int8_t* q, float* scale, std::uint32_t sources,
                                      std::uint32_t features, void* stream, char* err, int errlen) {
    return call(err, errlen,
                [&] { quantizeFeaturesInt8(x, q, scale, sources, features, static_cast<cudaStream_t>(stream)); });
}

EXPORT int ref_pack_features_int8x16(const std::int8_t* q, std::int8_t* packed, std::uint32_t sources,
                                     std::uint32_t features, void* stream, char* err, int errlen) {
    return call(err, errlen,
                [&] { packFeaturesInt8x16(q, packed, sources, features, static_cast<cudaStream_t>(stream)); });
}

EXPORT int ref_view_size(void) { return static_cast<int>(sizeof(Sw32DeviceView)); }
