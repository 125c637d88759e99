/*
 * ORACLE - test infrastructure, not product code.
 *
 * CPU restatement of the reference's arithmetic on the SpMM path (Shixg-cnic/tcc_spmm),
 * used only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as the
 * checker. The operators that are measured and shipped live in tcc_spmm_b200/csrc.
 *
 * Pinned by: the reference's own host code compiled from its sources into oracle/_ref
 * (format arrays, tasks, canonical CSR), the reference's own kernels run on the B200 (q,
 * scales, packed bytes, Y) and the golden fixtures under tests/golden made from both.
 *
 *   oracle_tf32_rna   cvt.rna.tf32.f32 of the PTX ISA (used at reference
 *                     src/kernel/spmm_kernel.cuh:7-11): round to 10 explicit mantissa bits,
 *                     ties away from zero, written as arithmetic on the exact value.
 *   oracle_quantize   reference src/format/int8_quantize.cu:4-25
 *   oracle_pack16     reference src/format/pack_int8.cu:6-15
 *   oracle_spmm       reference src/kernel/spmm_kernel.cuh:26-90,131-169,205-227: every
 *                     stored A value of a 32-row window times the dequantized source row,
 *                     tf32_rna(a) * tf32_rna(float(q) * scale), accumulated in FP32; padding
 *                     and out-of-range source slots contribute nothing. Optionally the
 *                     element-wise bound sum |a * q * scale| of the tolerance test.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define EXPORT __attribute__((visibility("default")))

EXPORT float oracle_tf32_rna(float x) {
    if (!isfinite(x) || x == 0.0f)
        return x;
    const double ax = fabs((double)x);
    int e2;
    frexp(ax, &e2); /* ax = f * 2^e2, f in [0.5, 1): floor(log2 ax) = e2 - 1 */
    int exponent = e2 - 1;
    if (exponent < -126)
        exponent = -126; /* subnormal FP32: fixed quantum */
    const double quantum = ldexp(1.0, exponent - 10);
    const double r = floor(ax / quantum + 0.5) * quantum;
    if (r >= ldexp(1.0, 128))
        return x > 0 ? INFINITY : -INFINITY;
    return (float)(x < 0 ? -r : r);
}

/* Same rounding on the bit pattern (add half an ulp of the 10-bit mantissa, clear the 13
 * dropped bits); the hot loops use it. Tests check it against oracle_tf32_rna. */
static inline float tf32_bits(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) /* Inf/NaN unchanged */
        return x;
    u = (u + 0x1000u) & 0xFFFFE000u;
    memcpy(&x, &u, 4);
    return x;
}

EXPORT float oracle_tf32_bits(float x) { return tf32_bits(x); }

EXPORT void oracle_tf32_rna_array(const float* in, float* out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i)
        out[i] = oracle_tf32_rna(in[i]);
}

EXPORT void oracle_quantize(const float* x, int8_t* q, float* scale, uint32_t sources, uint32_t features) {
    for (uint32_t r = 0; r < sources; ++r) {
        const float* xr = x + (uint64_t)r * features;
        float m = 0.0f;
        for (uint32_t j = 0; j < features; ++j)
            m = fmaxf(m, fabsf(xr[j]));
        const float s = m == 0.0f ? 1.0f : m / 127.f;
        scale[r] = s;
        for (uint32_t j = 0; j < features; ++j) {
            const int v = (int)lrintf(xr[j] / s);
            q[(uint64_t)r * features + j] = (int8_t)(v < -127 ? -127 : (v > 127 ? 127 : v));
        }
    }
}

EXPORT void oracle_pack16(const int8_t* q, int8_t* packed, uint32_t sources, uint32_t features) {
    const uint64_t tiles = (uint64_t)sources * features / 16;
    for (uint64_t t = 0; t < tiles; ++t)
        for (int i = 0; i < 8; ++i) {
            packed[16 * t + 2 * i] = q[16 * t + i];
            packed[16 * t + 2 * i + 1] = q[16 * t + i + 8];
        }
}

/*
 * Y rows of the listed windows: y[(w*32 + r)*F + f] for the w-th listed window `sw_list[w]`
 * and local row r (rows past `rows` stay zero). q is the unpacked INT8 matrix [cols][F].
 * bound (optional, same shape, double) receives sum |a * q * scale|.
 */
EXPORT int oracle_spmm(const uint32_t* window_offsets, const uint32_t* source_ids, const uint64_t* source_metadata,
                       const float* values, const int8_t* q, const float* scales, uint32_t rows, uint32_t cols,
                       uint32_t features, const uint32_t* sw_list, uint32_t sw_count, float* y, double* bound,
                       int threads) {
    if (features == 0 || features > 4096)
        return 1;
#ifdef _OPENMP
    if (threads > 0)
        omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        float* xh = (float*)malloc(sizeof(float) * features);
        double* xd = (double*)malloc(sizeof(double) * features);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (int64_t w = 0; w < (int64_t)sw_count; ++w) {
            const uint32_t sw = sw_list[w];
            float* yw = y + (uint64_t)w * 32 * features;
            double* bw = bound ? bound + (uint64_t)w * 32 * features : NULL;
            memset(yw, 0, sizeof(float) * 32 * features);
            if (bw)
                memset(bw, 0, sizeof(double) * 32 * features);
            for (uint32_t p = window_offsets[sw]; p < window_offsets[sw + 1]; ++p) {
                for (uint32_t k = 0; k < 8; ++k) {
                    const uint64_t slot = (uint64_t)p * 8 + k;
                    const uint32_t id = source_ids[slot];
                    const uint32_t mask = (uint32_t)source_metadata[slot];
                    const uint32_t first = (uint32_t)(source_metadata[slot] >> 32);
                    if (id >= cols || mask == 0)
                        continue;
                    const float s = scales[id];
                    const int8_t* qr = q + (uint64_t)id * features;
                    for (uint32_t f = 0; f < features; ++f) {
                        xh[f] = tf32_bits((float)qr[f] * s);
                        xd[f] = (double)qr[f] * (double)s;
                    }
                    uint32_t m = mask, j = 0;
                    while (m) {
                        const int r = __builtin_ctz(m);
                        m &= m - 1;
                        const float a = values[first + j];
                        const float at = tf32_bits(a);
                        ++j;
                        float* yr = yw + (uint64_t)r * features;
                        for (uint32_t f = 0; f < features; ++f)
                            yr[f] += at * xh[f];
                        if (bw) {
                            double* br = bw + (uint64_t)r * features;
                            for (uint32_t f = 0; f < features; ++f)
                                br[f] += fabs((double)a * xd[f]);
                        }
                    }
                }
            }
            if ((uint64_t)sw * 32 + 32 > rows) { /* rows past the matrix end */
                const uint32_t valid = rows - sw * 32;
                memset(yw + (uint64_t)valid * features, 0, sizeof(float) * (32 - valid) * features);
            }
        }
        free(xh);
        free(xd);
    }
    return 0;
}

EXPORT int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
