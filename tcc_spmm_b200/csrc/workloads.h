/* Seeded synthetic sparse matrices and features for tests and benchmarks
 * (libtcc_workloads). Not part of the SpMM operator boundary. Functions return 0 on
 * success, nonzero with tcc_wl_last_error() set otherwise. */
#ifndef TCC_WORKLOADS_H
#define TCC_WORKLOADS_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct tcc_wl_csr {
    uint32_t rows, cols;
    uint64_t nnz;
    uint32_t* rowOffsets; /* rows + 1 */
    uint32_t* sourceIds;  /* nnz, strictly increasing per row */
    float* values;        /* nnz, finite and nonzero */
} tcc_wl_csr;

const char* tcc_wl_last_error(void);
void tcc_wl_free(tcc_wl_csr* csr);

int tcc_wl_poisson(uint32_t rows, uint32_t cols, double mean, uint64_t seed, uint32_t threads, tcc_wl_csr** out);
int tcc_wl_powerlaw(uint32_t rows, uint64_t target_nnz, double alpha, uint32_t max_degree, double local_fraction,
                    uint32_t local_radius, uint64_t seed, uint32_t threads, tcc_wl_csr** out);
int tcc_wl_stress(uint32_t rows, uint32_t light_lo, uint32_t light_hi, uint32_t heavy_rows, uint32_t heavy_windows,
                  uint32_t heavy_lo, uint32_t heavy_hi, uint64_t seed, uint32_t threads, tcc_wl_csr** out);
int tcc_wl_rmat(uint32_t scale, uint64_t edges, double a, double b, double c, uint64_t seed, uint32_t threads,
                tcc_wl_csr** out);
/* count N(0,1) floats (Box-Muller). */
int tcc_wl_normal(float* out, uint64_t count, uint64_t seed, uint32_t threads);

/* The same R-MAT matrix as tcc_wl_rmat (bit for bit), generated on the current CUDA device in
 * device memory owned by the returned handle: the edge draws of every sampling block from the
 * same counter-based stream, a radix sort of (row, column) keys, duplicate removal, per-row
 * degrees and 1/deg_i values. `stream` is a cudaStream_t; the call returns once the arrays are
 * complete. Scratch of about 16 bytes per edge sample is allocated and freed inside the call. */
typedef struct tcc_wl_device_csr tcc_wl_device_csr;
int tcc_wl_rmat_device(uint32_t scale, uint64_t edges, double a, double b, double c, uint64_t seed, void* stream,
                       tcc_wl_device_csr** out);
/* Sizes and device arrays of a generated matrix (valid until tcc_wl_device_csr_free). */
int tcc_wl_device_csr_arrays(const tcc_wl_device_csr* csr, uint32_t* rows, uint32_t* cols, uint64_t* nnz,
                             uint32_t** row_offsets, uint32_t** source_ids, float** values);
void tcc_wl_device_csr_free(tcc_wl_device_csr* csr);

#ifdef __cplusplus
}
#endif
#endif
