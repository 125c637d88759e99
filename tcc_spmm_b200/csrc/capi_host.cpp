// extern "C" host entry points of libtcc_spmm_b200 (declared in include/tcc_spmm_b200.h).
#include "common.hpp"
#include "format/csr.h"
#include "format/sw32.h"

#include <cstring>
#include <string>

namespace tcc {
Sw32HostFormat convertCsr(std::uint32_t rows, std::uint32_t cols, const std::uint32_t* offsets,
                          const std::uint32_t* sources, const float* values, std::uint64_t nnz,
                          bool bucketed, unsigned threads);
CsrMatrix canonicalCsr(std::uint32_t rows, std::uint32_t cols, std::uint32_t nnz,
                       const std::uint32_t* offsets, const std::uint32_t* sources, const float* values,
                       unsigned threads);
MtxMatrix loadMatrixMarketFile(const std::string& path);
void partitionTasks(const tcc_sw32_task* tasks, std::uint32_t count, const std::uint32_t* masks,
                    std::uint32_t features, std::uint32_t parts, std::uint32_t* bounds);
void balanceTasks(const tcc_sw32_task* tasks, std::uint32_t count, const std::uint32_t* masks,
                  std::uint32_t features, std::uint32_t ctas, tcc_sw32_task* out);
std::uint32_t balanceTasksPadded(const tcc_sw32_task* tasks, std::uint32_t count, const std::uint32_t* masks,
                                 std::uint32_t features, std::uint32_t ctas, std::uint32_t ctasPerSm,
                                 tcc_sw32_task* out, std::uint64_t capacity);

namespace {
thread_local std::string lastError;
}
void setLastError(const std::string& message) { lastError = message; }
void clearLastError() { lastError.clear(); }

void throwStatus(int status, const char* message) {
    const std::string text = message ? message : "";
    switch (status) {
    case TCC_INVALID_ARGUMENT:
        throw std::invalid_argument(text);
    case TCC_OVERFLOW:
        throw std::overflow_error(text);
    default:
        throw std::runtime_error(text);
    }
}
} // namespace tcc

static_assert(sizeof(tcc_sw32_task) == 28, "Sw32Task ABI");
static_assert(sizeof(tcc_sw32_task) == sizeof(Sw32Task), "Sw32Task ABI");
static_assert(sizeof(tcc_sw32_reduce_range) == sizeof(Sw32ReduceRange), "Sw32ReduceRange ABI");
static_assert(sizeof(tcc_sw32_device_view) == sizeof(Sw32DeviceView), "Sw32DeviceView ABI");
static_assert(offsetof(tcc_sw32_device_view, taskCount) == offsetof(Sw32DeviceView, taskCount),
              "Sw32DeviceView ABI");

struct tcc_csr {
    std::uint32_t rows = 0;
    CsrMatrix csr;
};
struct tcc_sw32_host {
    Sw32HostFormat format;
};

extern "C" {

const char* tcc_last_error(void) { return tcc::lastError.c_str(); }

const char* tcc_version(void) { return "tcc-spmm-b200 0.1 (sm_100a)"; }

int tcc_make_canonical_csr(uint32_t rows, uint32_t cols, uint32_t nnz, const uint32_t* row_offsets,
                           const uint32_t* source_ids, const float* values, tcc_csr** out) {
    return tcc::guarded([&] {
        if (out == nullptr)
            throw std::invalid_argument("null output handle");
        *out = nullptr;
        auto* handle = new tcc_csr;
        try {
            handle->rows = rows;
            handle->csr = tcc::canonicalCsr(rows, cols, nnz, row_offsets, source_ids, values, 0);
        } catch (...) {
            delete handle;
            throw;
        }
        *out = handle;
    });
}

int tcc_csr_arrays(const tcc_csr* csr, uint32_t* rows, const uint32_t** row_offsets,
                   const uint32_t** source_ids, const float** values, uint64_t* nnz) {
    return tcc::guarded([&] {
        if (csr == nullptr)
            throw std::invalid_argument("null CSR handle");
        if (rows)
            *rows = csr->rows;
        if (row_offsets)
            *row_offsets = csr->csr.rowOffsets.data();
        if (source_ids)
            *source_ids = csr->csr.sourceIds.data();
        if (values)
            *values = csr->csr.values.data();
        if (nnz)
            *nnz = csr->csr.sourceIds.size();
    });
}

void tcc_csr_free(tcc_csr* csr) { delete csr; }

int tcc_load_matrix_market(const char* path, uint32_t* cols, tcc_csr** out) {
    return tcc::guarded([&] {
        if (path == nullptr || out == nullptr)
            throw std::invalid_argument("null path or output handle");
        *out = nullptr;
        auto* handle = new tcc_csr;
        try {
            MtxMatrix m = tcc::loadMatrixMarketFile(path);
            handle->rows = m.rows;
            handle->csr = std::move(m.csr);
            if (cols)
                *cols = m.cols;
        } catch (...) {
            delete handle;
            throw;
        }
        *out = handle;
    });
}

int tcc_convert_csr_to_sw32(uint32_t rows, uint32_t cols, const uint32_t* row_offsets,
                            const uint32_t* source_ids, const float* values, uint64_t nnz,
                            int bucket_by_rw_mask, uint32_t threads, tcc_sw32_host** out) {
    return tcc::guarded([&] {
        if (out == nullptr)
            throw std::invalid_argument("null output handle");
        *out = nullptr;
        auto* handle = new tcc_sw32_host;
        try {
            handle->format = tcc::convertCsr(rows, cols, row_offsets, source_ids, values, nnz,
                                             bucket_by_rw_mask != 0, threads);
        } catch (...) {
            delete handle;
            throw;
        }
        *out = handle;
    });
}

int tcc_sw32_host_sizes(const tcc_sw32_host* host, tcc_sw32_sizes* sizes) {
    return tcc::guarded([&] {
        if (host == nullptr || sizes == nullptr)
            throw std::invalid_argument("null SW32 handle");
        const auto& f = host->format;
        sizes->rows = f.rows;
        sizes->cols = f.cols;
        sizes->partialCount = f.partialCount;
        sizes->bucketed = f.bucketOffsets.empty() ? 0u : 1u;
        sizes->windowOffsets = f.windowOffsets.size();
        sizes->sourceIds = f.sourceIds.size();
        sizes->rowGroupMasks = f.rowGroupMasks.size();
        sizes->values = f.values.size();
        sizes->bucketOffsets = f.bucketOffsets.size();
        sizes->tasks = f.tasks.size();
        sizes->reductions = f.reductions.size();
        sizes->partialIds = f.partialIds.size();
    });
}

int tcc_sw32_host_arrays(const tcc_sw32_host* host, tcc_sw32_arrays* arrays) {
    return tcc::guarded([&] {
        if (host == nullptr || arrays == nullptr)
            throw std::invalid_argument("null SW32 handle");
        const auto& f = host->format;
        arrays->windowOffsets = f.windowOffsets.data();
        arrays->sourceIds = f.sourceIds.data();
        arrays->rowGroupMasks = f.rowGroupMasks.data();
        arrays->sourceMetadata = f.sourceMetadata.data();
        arrays->values = f.values.data();
        arrays->bucketOffsets = f.bucketOffsets.data();
        arrays->tasks = reinterpret_cast<const tcc_sw32_task*>(f.tasks.data());
        arrays->reductions = reinterpret_cast<const tcc_sw32_reduce_range*>(f.reductions.data());
        arrays->partialIds = f.partialIds.data();
    });
}

void tcc_sw32_host_free(tcc_sw32_host* host) { delete host; }

int tcc_partition_tasks(const tcc_sw32_task* tasks, uint32_t task_count, const uint32_t* row_group_masks,
                        uint32_t features, uint32_t parts, uint32_t* bounds) {
    return tcc::guarded([&] {
        if (bounds == nullptr)
            throw std::invalid_argument("null bounds");
        tcc::partitionTasks(tasks, task_count, row_group_masks, features, parts, bounds);
    });
}

int tcc_balance_tasks(const tcc_sw32_task* tasks, uint32_t task_count, const uint32_t* row_group_masks,
                      uint32_t features, uint32_t ctas, tcc_sw32_task* out) {
    return tcc::guarded([&] {
        if (out == tasks && task_count != 0)
            throw std::invalid_argument("out must not alias tasks");
        tcc::balanceTasks(tasks, task_count, row_group_masks, features, ctas, out);
    });
}

int tcc_balance_tasks_padded(const tcc_sw32_task* tasks, uint32_t task_count, const uint32_t* row_group_masks,
                             uint32_t features, uint32_t ctas, uint32_t ctas_per_sm, tcc_sw32_task* out,
                             uint64_t out_capacity, uint32_t* out_count) {
    return tcc::guarded([&] {
        if (out_count == nullptr)
            throw std::invalid_argument("out_count must not be null");
        if (out != nullptr && out == tasks && task_count != 0)
            throw std::invalid_argument("out must not alias tasks");
        *out_count = tcc::balanceTasksPadded(tasks, task_count, row_group_masks, features, ctas, ctas_per_sm, out,
                                             out_capacity);
    });
}

int tcc_spmm_workspace_size(uint32_t rows, uint32_t partial_count, uint32_t features,
                            uint64_t* partial_floats, uint64_t* counter_words) {
    return tcc::guarded([&] {
        if (features != 128 && features != 256)
            throw std::invalid_argument("feature dimension must be 128 or 256");
        const uint64_t windows = (uint64_t(rows) + 31) / 32;
        if (partial_floats)
            *partial_floats = uint64_t(partial_count) * 8 * features;
        if (counter_words)
            *counter_words = partial_count ? windows * (features / 128) : 0;
    });
}

} // extern "C"
