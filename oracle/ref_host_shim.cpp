// ORACLE - test infrastructure, not product code.
// extern "C" wrapper around the reference's own host code (Shixg-cnic/tcc_spmm
// src/format/sw32.cpp, csr.cpp, matrix_market.cpp), compiled from the reference sources
// where they lie into oracle/_ref/libtcc_ref_host.so by oracle/build.py. Everything except
// the ref_* functions is hidden, so this library never interposes the product's symbols.
#include "format/csr.h"
#include "format/sw32.h"

#include <cstring>
#include <new>
#include <stdexcept>
#include <string>

#define EXPORT extern "C" __attribute__((visibility("default")))

namespace {
int fail(const std::exception& e, int code, char* err, int errlen) {
    if (err && errlen > 0) {
        std::strncpy(err, e.what(), errlen - 1);
        err[errlen - 1] = '\0';
    }
    return code;
}
template <typename Body> int call(char* err, int errlen, Body&& body) {
    try {
        body();
        return 0;
    } catch (const std::invalid_argument& e) {
        return fail(e, 1, err, errlen);
    } catch (const std::overflow_error& e) {
        return fail(e, 2, err, errlen);
    } catch (const std::runtime_error& e) {
        return fail(e, 3, err, errlen);
    } catch (const std::exception& e) {
        return fail(e, 4, err, errlen);
    }
}
struct RefCsr {
    std::uint32_t rows = 0, cols = 0;
    CsrMatrix csr;
};
} // namespace

EXPORT int ref_convert_csr_to_sw32(std::uint32_t rows, std::uint32_t cols, const std::uint32_t* rowOffsets,
                                   std::uint64_t offsetCount, const std::uint32_t* sourceIds, const float* values,
                                   std::uint64_t nnz, int bucketed, void** out, char* err, int errlen) {
    return call(err, errlen, [&] {
        CsrMatrix csr;
        csr.rowOffsets.assign(rowOffsets, rowOffsets + offsetCount);
        csr.sourceIds.assign(sourceIds, sourceIds + nnz);
        csr.values.assign(values, values + nnz);
        *out = new Sw32HostFormat(convertCsrToSw32(rows, cols, csr, bucketed != 0));
    });
}

// sizes[0..8]: windowOffsets, sourceIds, rowGroupMasks, sourceMetadata, values,
// bucketOffsets, tasks, reductions, partialIds; sizes[9] = partialCount.
EXPORT void ref_sw32_sizes(const void* handle, std::uint64_t* sizes) {
    const auto& f = *static_cast<const Sw32HostFormat*>(handle);
    sizes[0] = f.windowOffsets.size();
    sizes[1] = f.sourceIds.size();
    sizes[2] = f.rowGroupMasks.size();
    sizes[3] = f.sourceMetadata.size();
    sizes[4] = f.values.size();
    sizes[5] = f.bucketOffsets.size();
    sizes[6] = f.tasks.size();
    sizes[7] = f.reductions.size();
    sizes[8] = f.partialIds.size();
    sizes[9] = f.partialCount;
}

EXPORT void ref_sw32_arrays(const void* handle, const void** arrays) {
    const auto& f = *static_cast<const Sw32HostFormat*>(handle);
    arrays[0] = f.windowOffsets.data();
    arrays[1] = f.sourceIds.data();
    arrays[2] = f.rowGroupMasks.data();
    arrays[3] = f.sourceMetadata.data();
    arrays[4] = f.values.data();
    arrays[5] = f.bucketOffsets.data();
    arrays[6] = f.tasks.data();
    arrays[7] = f.reductions.data();
    arrays[8] = f.partialIds.data();
}

EXPORT void ref_sw32_free(void* handle) { delete static_cast<Sw32HostFormat*>(handle); }

EXPORT int ref_make_canonical_csr(std::uint32_t rows, std::uint32_t cols, std::uint32_t nnz,
                                  const std::uint32_t* rowOffsets, const std::uint32_t* sourceIds,
                                  const float* values, void** out, char* err, int errlen) {
    return call(err, errlen, [&] {
        auto* r = new RefCsr;
        try {
            r->rows = rows;
            r->cols = cols;
            r->csr = makeCanonicalCsr(rows, cols, nnz, rowOffsets, sourceIds, values);
        } catch (...) {
            delete r;
            throw;
        }
        *out = r;
    });
}

EXPORT int ref_load_matrix_market(const char* path, void** out, char* err, int errlen) {
    return call(err, errlen, [&] {
        MtxMatrix m = loadMatrixMarket(path);
        auto* r = new RefCsr;
        r->rows = m.rows;
        r->cols = m.cols;
        r->csr = std::move(m.csr);
        *out = r;
    });
}

// dims[0] = rows, dims[1] = cols, dims[2] = nnz; arrays = rowOffsets, sourceIds, values.
EXPORT void ref_csr_view(const void* handle, std::uint64_t* dims, const void** arrays) {
    const auto& r = *static_cast<const RefCsr*>(handle);
    dims[0] = r.rows;
    dims[1] = r.cols;
    dims[2] = r.csr.sourceIds.size();
    arrays[0] = r.csr.rowOffsets.data();
    arrays[1] = r.csr.sourceIds.data();
    arrays[2] = r.csr.values.data();
}

EXPORT void ref_csr_free(void* handle) { delete static_cast<RefCsr*>(handle); }
