/*
 * C ABI of tcc-spmm-b200: the fused Y = A x dequant(X_int8) SpMM for B200 (sm_100a).
 *
 * Every entry point returns a tcc_status. A nonzero status comes with a message that
 * tcc_last_error() returns on the same host thread. No C++ exception crosses this
 * boundary. The C++ drop-in headers (spmm.cuh, format/sw32.h, ...) wrap these functions and turn
 * the status back into the exception type that the reference API throws.
 *
 * Conventions shared with the reference library (Shixg-cnic/tcc_spmm):
 *   - The caller allocates and owns every device buffer. Device entry points allocate
 *     nothing and never synchronise; they enqueue work on `stream` and return. The one
 *     exception is the device format builder (tcc_convert_csr_to_sw32_device), whose output
 *     sizes depend on the data.
 *   - Sizes are 32-bit, as in the reference (rows, cols, features, nnz).
 *   - All device pointers are plain CUDA device addresses; `stream` is a cudaStream_t
 *     (NULL = legacy default stream).
 */
#ifndef TCC_SPMM_B200_H
#define TCC_SPMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in cuda_runtime.h. */
typedef struct CUstream_st* tcc_stream_t;

typedef enum tcc_status {
    TCC_OK = 0,
    TCC_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
    TCC_OVERFLOW = 2,         /* reference: std::overflow_error    */
    TCC_CUDA_ERROR = 3,       /* reference: std::runtime_error (checkCuda) */
    TCC_INTERNAL = 4,         /* any other failure (allocation on the host, ...) */
    TCC_DEVICE_TIMEOUT = 5    /* a bounded device wait ran out (see tcc_device_status) */
} tcc_status;

/* Sw32Task, 7 x u32 = 28 bytes (include/format/sw32.h:13-15 in the reference). */
typedef struct tcc_sw32_task {
    uint32_t sw, begin, end, partial, mask, chunks, reduceFirst;
} tcc_sw32_task;

/* Sw32ReduceRange (include/format/sw32.h:16-18). */
typedef struct tcc_sw32_reduce_range {
    uint32_t begin, end;
} tcc_sw32_reduce_range;

/* Sw32DeviceView, byte-compatible (include/format/sw32.h:47-56): nine device pointers
 * followed by the task count. */
typedef struct tcc_sw32_device_view {
    const uint32_t* windowOffsets;
    const uint32_t* sourceIds;
    const uint32_t* rowGroupMasks;
    const uint64_t* sourceMetadata;
    const float* values;
    const uint32_t* bucketOffsets;
    const tcc_sw32_task* tasks;
    const tcc_sw32_reduce_range* reductions;
    const uint32_t* partialIds;
    uint32_t taskCount;
} tcc_sw32_device_view;

/* Message of the last failed call on this host thread ("" if none). */
const char* tcc_last_error(void);

/* Library version string. */
const char* tcc_version(void);

/* ---------------------------------------------------------------------------------
 * Device entry points
 * --------------------------------------------------------------------------------- */

/* Replaces launchSpmmInt8 (reference include/spmm.cuh:21-23, src/kernel/spmm.cu:17-31).
 * Y[rows x features] = A x (q * scale), A given by the uploaded SW32 view, packed_x the
 * packed16 INT8 features [cols x features], scales one float per source row.
 * features must be 128 or 256 (else TCC_INVALID_ARGUMENT, as the reference throws
 * std::invalid_argument). partials = partialCount*8*features floats and counters =
 * ceil(rows/32)*(features/128) u32 (zero before the first use, zero again after each
 * launch); both may be NULL when partialCount is 0. Every Y element is overwritten.
 * Launches on distinct workspaces may run concurrently. */
int tcc_launch_spmm_int8(const tcc_sw32_device_view* matrix, const int8_t* packed_x,
                         const float* scales, float* output, uint32_t rows, uint32_t cols,
                         uint32_t features, float* partials, uint32_t* counters,
                         tcc_stream_t stream);

/* Replaces quantizeFeaturesInt8 (reference include/format/int8_features.cuh:9-10,
 * src/format/int8_quantize.cu:27-31). Per source row: scale = absmax/127 (1 when the row
 * is all zero), q = clamp(lrintf(x/scale), -127, 127). Byte-identical to the reference. */
int tcc_quantize_features_int8(const float* x, int8_t* q, float* scale, uint32_t sources,
                               uint32_t features, tcc_stream_t stream);

/* Replaces packFeaturesInt8x16 (reference include/format/int8_features.cuh:14-15,
 * src/format/pack_int8.cu:18-25): every 16-feature tile becomes [q0,q8,q1,q9,...,q7,q15].
 * features % 16 == 0, packed must not alias q. Byte-identical to the reference. */
int tcc_pack_features_int8x16(const int8_t* q, int8_t* packed, uint32_t sources,
                              uint32_t features, tcc_stream_t stream);

/* One-pass quantize + pack: reads x once and writes the packed16 bytes and the scales
 * that quantizeFeaturesInt8 followed by packFeaturesInt8x16 would write (byte-identical).
 * No separate reference entry point; it fuses reference src/format/int8_quantize.cu:4-25
 * and src/format/pack_int8.cu:6-15. features % 16 == 0. */
int tcc_quantize_pack_features_int8(const float* x, int8_t* packed, float* scale,
                                    uint32_t sources, uint32_t features, tcc_stream_t stream);

/* Workspace sizing of reference src/device_matrix.cuh:18-28: partial floats
 * (partialCount*8*features) and counter words (ceil(rows/32)*(features/128), 0 when
 * partialCount is 0). */
int tcc_spmm_workspace_size(uint32_t rows, uint32_t partial_count, uint32_t features,
                            uint64_t* partial_floats, uint64_t* counter_words);

/* tcc_launch_spmm_int8 without a caller-provided workspace: the split-window partials and
 * counters live in a static device scratch of this library (8 MiB of partials, i.e.
 * partial_count * 8 * features <= 2^21 floats, and 1 MiB of counters, i.e.
 * ceil(rows / 32) * features / 128 <= 2^18 words); larger needs return
 * TCC_INVALID_ARGUMENT. partial_count must be the format's partialCount: the view does not
 * carry it, and a smaller value lets split tasks write past the checked size (undefined).
 * The library allocates nothing: the first call on a device looks up the scratch's address
 * (do it before any stream capture). The counters start at zero and every completed call
 * leaves them at zero; after a call whose bounded wait ran out, tcc_device_status(&s, 1)
 * returns them to zero. Calls on one device share the scratch, so they must not overlap
 * (serialise them on one stream). No counterpart in the reference, whose launchSpmmInt8
 * always takes the caller's SpmmWorkspace (include/spmm.cuh:10-23). */
int tcc_launch_spmm_int8_static_workspace(const tcc_sw32_device_view* matrix, const int8_t* packed_x,
                                          const float* scales, float* output, uint32_t rows,
                                          uint32_t cols, uint32_t features, uint32_t partial_count,
                                          tcc_stream_t stream);

/* Status word of the SpMM kernels on the current device since the last reset: bit 0 = a
 * bounded device wait ran out (the launch returned early, Y is incomplete, and the tickets of
 * split windows may be left short of zero), bit 1 = a split task found no partial/counter
 * workspace (its rows were not written). Synchronises the device. reset != 0 clears the word
 * and returns the static workspace's counters to zero; counters in a caller's workspace are
 * the caller's to re-zero (cudaMemset) after bit 0. No counterpart in the reference, whose
 * kernel has no bounded waits. */
int tcc_device_status(uint32_t* status, int reset);

/* ---------------------------------------------------------------------------------
 * Host format construction (no GPU needed)
 * --------------------------------------------------------------------------------- */

/* Canonical CSR owned by the library (reference include/format/csr.h:7-10). */
typedef struct tcc_csr tcc_csr;

/* Replaces makeCanonicalCsr (reference include/format/csr.h:23-25,
 * src/format/csr.cpp:6-40): stable-sort each row by column, sum duplicates in that order,
 * drop zero sums, reject non-finite values and invalid offsets. */
int tcc_make_canonical_csr(uint32_t rows, uint32_t cols, uint32_t nnz,
                           const uint32_t* row_offsets, const uint32_t* source_ids,
                           const float* values, tcc_csr** out);
/* Views into a tcc_csr (valid until tcc_csr_free). row_offsets has rows+1 entries. */
int tcc_csr_arrays(const tcc_csr* csr, uint32_t* rows, const uint32_t** row_offsets,
                   const uint32_t** source_ids, const float** values, uint64_t* nnz);
void tcc_csr_free(tcc_csr* csr);

/* Replaces loadMatrixMarket (reference include/format/csr.h:18,
 * src/format/matrix_market.cpp:30-103): coordinate real/integer/pattern,
 * general/symmetric, symmetric off-diagonals mirrored, then makeCanonicalCsr. The row count
 * is available through tcc_csr_arrays; cols receives the column count. File and format
 * errors return TCC_INTERNAL (the reference throws std::runtime_error). */
int tcc_load_matrix_market(const char* path, uint32_t* cols, tcc_csr** out);

/* SW32 host format owned by the library (reference include/format/sw32.h:22-39). */
typedef struct tcc_sw32_host tcc_sw32_host;

typedef struct tcc_sw32_sizes {
    uint32_t rows, cols, partialCount, bucketed;
    uint64_t windowOffsets;  /* windows + 1 */
    uint64_t sourceIds;      /* 8 * panels (== sourceMetadata) */
    uint64_t rowGroupMasks;  /* panels */
    uint64_t values;         /* nnz */
    uint64_t bucketOffsets;  /* 17 * windows, or 0 when not bucketed */
    uint64_t tasks, reductions, partialIds;
} tcc_sw32_sizes;

typedef struct tcc_sw32_arrays {
    const uint32_t* windowOffsets;
    const uint32_t* sourceIds;
    const uint32_t* rowGroupMasks;
    const uint64_t* sourceMetadata;
    const float* values;
    const uint32_t* bucketOffsets;
    const tcc_sw32_task* tasks;
    const tcc_sw32_reduce_range* reductions;
    const uint32_t* partialIds;
} tcc_sw32_arrays;

/* Replaces convertCsrToSw32 (reference include/format/sw32.h:43-44,
 * src/format/sw32.cpp:69-167) including buildPanelTasks (src/format/sw32.cpp:25-65).
 * Output arrays are byte-identical to the reference; the conversion runs on `threads`
 * host threads (0 = all hardware threads). */
int tcc_convert_csr_to_sw32(uint32_t rows, uint32_t cols, const uint32_t* row_offsets,
                            const uint32_t* source_ids, const float* values, uint64_t nnz,
                            int bucket_by_rw_mask, uint32_t threads, tcc_sw32_host** out);
int tcc_sw32_host_sizes(const tcc_sw32_host* host, tcc_sw32_sizes* sizes);
int tcc_sw32_host_arrays(const tcc_sw32_host* host, tcc_sw32_arrays* arrays);
void tcc_sw32_host_free(tcc_sw32_host* host);

/* ---------------------------------------------------------------------------------
 * Upload of a host format
 * --------------------------------------------------------------------------------- */

/* A host SW32 format uploaded to one device together with its split-task workspace, owned by
 * the library. */
typedef struct tcc_device_matrix tcc_device_matrix;

/* Replaces the constructor of the reference's DeviceMatrix (src/device_matrix.cuh:18-28):
 * copies every array of a host SW32 format (sizes and host pointers as tcc_sw32_host_sizes and
 * tcc_sw32_host_arrays give them, or a caller's own arrays laid out the same way) to the current
 * device and sizes the workspace for `features` (128 or 256): partials = partialCount * 8 *
 * features floats and counters = windows * (features / 128) u32 set to zero, both only when
 * partialCount > 0 (NULL otherwise). One device allocation holds everything, each array 256-byte
 * aligned. The copies run on `stream`, which is synchronised before the call returns, so the host
 * arrays may be released afterwards. Unlike the launch entry points this call allocates. */
int tcc_device_matrix_upload(const tcc_sw32_sizes* sizes, const tcc_sw32_arrays* arrays,
                             uint32_t features, tcc_stream_t stream, tcc_device_matrix** out);
/* view() and workspace() of the reference's DeviceMatrix (src/device_matrix.cuh:30-37): the
 * device view of all tasks and the partial/counter pointers (NULL when partialCount is 0). */
int tcc_device_matrix_view(const tcc_device_matrix* matrix, tcc_sw32_device_view* view);
int tcc_device_matrix_workspace(const tcc_device_matrix* matrix, float** partials,
                                uint32_t** counters);
/* Frees the device memory (the reference's DeviceBuffer destructors). */
void tcc_device_matrix_free(tcc_device_matrix* matrix);

/* ---------------------------------------------------------------------------------
 * Device format construction
 * --------------------------------------------------------------------------------- */

/* SW32 format built on the GPU, owned by the library (one device allocation). */
typedef struct tcc_sw32_device tcc_sw32_device;

/* convertCsrToSw32 (reference include/format/sw32.h:43-44, src/format/sw32.cpp:69-167) and
 * buildPanelTasks (src/format/sw32.cpp:25-65) on the current device, from a canonical CSR
 * whose row_offsets (rows + 1), source_ids and values (nnz each) are device pointers. The
 * arrays are byte-identical to tcc_convert_csr_to_sw32's, and invalid input gives the same
 * status and message. No reference counterpart: the reference builds the format on the host
 * only. Unlike the launch entry points this call allocates device memory and synchronises
 * `stream` a few times to read sizes; the arrays are ready for work enqueued on `stream` after
 * it returns. Its memory (the output, and scratch of at most about 36 bytes per nonzero that is
 * released in stream order before the call returns) comes from a memory pool of the library,
 * one per device, that keeps freed memory for the next build until tcc_sw32_device_trim. */
int tcc_convert_csr_to_sw32_device(uint32_t rows, uint32_t cols, const uint32_t* row_offsets,
                                   const uint32_t* source_ids, const float* values, uint64_t nnz,
                                   int bucket_by_rw_mask, tcc_stream_t stream, tcc_sw32_device** out);
/* Sizes and device pointers of the built arrays (valid until tcc_sw32_device_free). Every
 * pointer is non-null, also for an empty array. */
int tcc_sw32_device_sizes(const tcc_sw32_device* format, tcc_sw32_sizes* sizes);
int tcc_sw32_device_arrays(const tcc_sw32_device* format, tcc_sw32_arrays* arrays);
/* The device view of all tasks, as an upload would give it (reference
 * src/device_matrix.cuh:8-37 builds the same view from its uploaded arrays). */
int tcc_sw32_device_view_of(const tcc_sw32_device* format, tcc_sw32_device_view* view);
/* Frees the arrays into the library's pool (synchronises the device). */
void tcc_sw32_device_free(tcc_sw32_device* format);
/* Returns the memory that the library's pool of the current device holds unused. */
int tcc_sw32_device_trim(void);

/* Multi-GPU sharding (no reference counterpart; the reference is single-GPU): cut the
 * task array into `parts` contiguous ranges at SW boundaries with balanced estimated cost
 * (panels, active row-group MMAs and the per-task write-back). bounds gets parts+1 task
 * indices, bounds[0] = 0 and bounds[parts] = task_count. Every split SW stays on one
 * part, so its partials, counter and merge are local to one GPU. */
int tcc_partition_tasks(const tcc_sw32_task* tasks, uint32_t task_count,
                        const uint32_t* row_group_masks, uint32_t features, uint32_t parts,
                        uint32_t* bounds);

/* Task order for one launch (no reference counterpart; the reference launches one CTA per task):
 * the fast-path kernels are persistent, CTA b of a grid of G = min(ctas, task_count) CTAs taking
 * tasks b, b + G, b + 2G, ... of the view. out receives a permutation of tasks that deals them
 * heaviest first (the cost estimate of tcc_partition_tasks), one per CTA per round, to the CTA
 * with the least work so far, so that the CTAs finish together. Y is bit-identical for any task
 * order. ctas = the grid of the launch (tcc_spmm_launch_shape); out must not alias tasks. */
int tcc_balance_tasks(const tcc_sw32_task* tasks, uint32_t task_count, const uint32_t* row_group_masks,
                      uint32_t features, uint32_t ctas, tcc_sw32_task* out);

/* Task order for one launch of the default kernel, weighted by resident-CTA speed (no reference
 * counterpart): as tcc_balance_tasks, but the tasks go heaviest first to the CTA that would
 * finish them earliest, the k-th resident CTA of an SM counting at its measured relative speed
 * (the SM's schedulers favour older CTAs; CTA b of a full grid of `ctas` CTAs, `ctas_per_sm` per
 * SM, is the (b / (ctas / ctas_per_sm))-th). CTAs then take different numbers of tasks: CTA b's
 * list sits at entries b, b + G, ... (G = min(ctas, task_count)), and shorter lists are padded
 * with entries of window 0xFFFFFFFF (no panels, no rows), which every kernel skips. *out_count
 * receives the number of entries, G * (longest list); with out == NULL only the count is
 * returned, else out_capacity must hold it. Y is bit-identical for any such order. */
int tcc_balance_tasks_padded(const tcc_sw32_task* tasks, uint32_t task_count, const uint32_t* row_group_masks,
                             uint32_t features, uint32_t ctas, uint32_t ctas_per_sm, tcc_sw32_task* out,
                             uint64_t out_capacity, uint32_t* out_count);

/* Launch shape of an SpMM kernel variant on the current device (variant 0 = what
 * tcc_launch_spmm_int8 runs on 16-byte aligned arrays): grid (persistent CTAs; 0 for the
 * per-task generic kernel), threads per CTA, dynamic shared memory and resident CTAs per SM. */
int tcc_spmm_launch_shape(uint32_t features, int variant, uint32_t* grid, uint32_t* threads, uint32_t* smem,
                          int* occupancy);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* TCC_SPMM_B200_H */
