/*
 * spmm_oracle.h -- CPU restatement of the reference's BOO / PBR builders and
 * CPU SpMM (Dayan135/SPMM, package torch_fast_spdmm).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (spmm_b200/, include/)
 * links, loads or calls this code.  It is the checker that the CUDA path is
 * compared against; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg use it.
 *
 * Parity is pinned two ways (see tests/test_oracle_pin.py):
 *   - against the reference's own C++ core compiled from its sources into
 *     oracle/_ref/ (oracle/build_ref.py), on seeded inputs: every format array
 *     bit-exact, CPU SpMM results bit-exact;
 *   - against committed golden fixtures in tests/golden/ generated from that
 *     same reference build by tests/golden/gen_golden.py.
 *
 * Index arrays are int64 here regardless of the reference's index_t; values
 * are float or double (functions come in _f32 / _f64 pairs).  All output
 * arrays are malloc'd by the oracle and released with the matching _free.
 *
 * Known, documented limits of the restatement (inputs the reference itself
 * leaves implementation-defined):
 *   - the remainder rows are sorted by (col, value) with qsort; two entries
 *     with equal column and values that compare equal but differ in bits
 *     (+0.0 / -0.0) or NaN values may land in a different order than the
 *     reference's std::sort puts them.
 *   - PBR blocks are emitted in canonical (stripe, block column) order; the
 *     reference emits them per stripe in std::unordered_map iteration order
 *     (pbr_matrix.cpp:396).  oracle_pbr_matmul_* takes the arrays as given, so
 *     it reproduces the reference's result for either order.
 */
#ifndef SPMM_ORACLE_H
#define SPMM_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ORACLE_OK = 0,
    ORACLE_ELABEL = 1,      /* cluster label out of range (boo_matrix.cpp:31-33) */
    ORACLE_EU16 = 2,        /* block local index space exceeds uint16 (:154-159) */
    ORACLE_EMERGE = 3,      /* 'merge' policy rejected (:65-76) */
    ORACLE_EPOLICY = 4,     /* unknown small_block_policy (:77-80) */
    ORACLE_EORDER = 5,      /* unknown nz_order (:81-83) */
    ORACLE_ELABELLEN = 6,   /* label array length mismatch (:91-94) */
    ORACLE_ENOMEM = 7
};

typedef struct {
    int64_t rows, cols, total_nnz;
    int64_t n_rg, n_cg, nb, nnz_c, rem_nnz, tail_nnz;
    int64_t max_nr, max_nc, max_nnz_blk;
    int32_t nz_order;
    int32_t scalar_size;          /* 4 or 8 */
    int64_t *row_grp_ptr, *row_ids, *col_grp_ptr, *col_ids;
    int64_t *blk_row_grp, *blk_col_grp, *blk_nz_ptr;
    uint8_t *blk_shift;
    uint16_t *nz_idx;
    void *nz_val;
    int64_t *rem_indptr, *rem_col_ind;
    void *rem_vals;
    int64_t *tail_row, *tail_col;
    void *tail_val;
} oracle_boo;

typedef struct {
    int64_t rows, cols, block_rows, block_cols, total_nnz;
    int64_t nb, nnz_c, rem_nnz;
    int32_t scalar_size;
    uint64_t *codes;              /* nb */
    int64_t *coords;              /* 2*nb, (row, col) of each block's top-left */
    int64_t *offsets;             /* nb+1 */
    void *data;                   /* nnz_c */
    int64_t *rem_indptr, *rem_col_ind;
    void *rem_vals;
} oracle_pbr;

/* boo_matrix.cpp:53-274 */
int oracle_csr_to_boo_f32(int64_t rows, int64_t cols, int64_t nnz, const int64_t *indptr,
                          const int64_t *indices, const float *data, const int32_t *row_labels,
                          int64_t n_row_labels, const int32_t *col_labels, int64_t n_col_labels,
                          int policy, int64_t threshold, int nz_order, oracle_boo *out);
int oracle_csr_to_boo_f64(int64_t rows, int64_t cols, int64_t nnz, const int64_t *indptr,
                          const int64_t *indices, const double *data, const int32_t *row_labels,
                          int64_t n_row_labels, const int32_t *col_labels, int64_t n_col_labels,
                          int policy, int64_t threshold, int nz_order, oracle_boo *out);
void oracle_boo_free(oracle_boo *b);

/* boo_matrix.cpp:336-396.  Y[batch][rows][K] is overwritten (zeroed first). */
void oracle_boo_matmul_f32(int64_t rows, int64_t cols, int64_t nb, const int64_t *row_grp_ptr,
                           const int64_t *row_ids, const int64_t *col_grp_ptr,
                           const int64_t *col_ids, const int64_t *blk_row_grp,
                           const int64_t *blk_col_grp, const int64_t *blk_nz_ptr,
                           const uint8_t *blk_shift, const uint16_t *nz_idx, const float *nz_val,
                           const int64_t *rem_indptr, const int64_t *rem_col_ind,
                           const float *rem_vals, int64_t tail_nnz, const int64_t *tail_row,
                           const int64_t *tail_col, const float *tail_val, const float *x,
                           int64_t batch, int64_t K, float *y);
void oracle_boo_matmul_f64(int64_t rows, int64_t cols, int64_t nb, const int64_t *row_grp_ptr,
                           const int64_t *row_ids, const int64_t *col_grp_ptr,
                           const int64_t *col_ids, const int64_t *blk_row_grp,
                           const int64_t *blk_col_grp, const int64_t *blk_nz_ptr,
                           const uint8_t *blk_shift, const uint16_t *nz_idx, const double *nz_val,
                           const int64_t *rem_indptr, const int64_t *rem_col_ind,
                           const double *rem_vals, int64_t tail_nnz, const int64_t *tail_row,
                           const int64_t *tail_col, const double *tail_val, const double *x,
                           int64_t batch, int64_t K, double *y);

/* boo_matrix.cpp:277-333: writes indptr[rows+1], indices[total], data[total]. */
void oracle_boo_to_csr_f32(const oracle_boo *b, int64_t *indptr, int64_t *indices, float *data);
void oracle_boo_to_csr_f64(const oracle_boo *b, int64_t *indptr, int64_t *indices, double *data);

/* pbr_matrix.cpp:333-448, blocks in canonical (stripe, block column) order.
 * min_nnz_per_block follows the reference's uint8_t parameter. */
int oracle_csr_to_pbr_f32(int64_t rows, int64_t cols, int64_t nnz, const int64_t *indptr,
                          const int64_t *indices, const float *data, int64_t block_rows,
                          int64_t block_cols, uint8_t min_nnz_per_block, oracle_pbr *out);
int oracle_csr_to_pbr_f64(int64_t rows, int64_t cols, int64_t nnz, const int64_t *indptr,
                          const int64_t *indices, const double *data, int64_t block_rows,
                          int64_t block_cols, uint8_t min_nnz_per_block, oracle_pbr *out);
void oracle_pbr_free(oracle_pbr *p);

/* pbr_matrix.cpp:17-68.  Consumes block data in bit order, block by block in
 * the order given.  Y[batch][rows][K] is overwritten. */
void oracle_pbr_matmul_f32(int64_t rows, int64_t cols, int64_t block_rows, int64_t block_cols,
                           int64_t nb, const uint64_t *codes, const int64_t *coords,
                           const float *data, const int64_t *rem_indptr,
                           const int64_t *rem_col_ind, const float *rem_vals, const float *x,
                           int64_t batch, int64_t K, float *y);
void oracle_pbr_matmul_f64(int64_t rows, int64_t cols, int64_t block_rows, int64_t block_cols,
                           int64_t nb, const uint64_t *codes, const int64_t *coords,
                           const double *data, const int64_t *rem_indptr,
                           const int64_t *rem_col_ind, const double *rem_vals, const double *x,
                           int64_t batch, int64_t K, double *y);

/* pbr_matrix.cpp:279-331 (rows' entries sorted by (col, value)). Returns 0, or
 * 1 when a block has a bit set past the last matrix row. */
int oracle_pbr_to_csr_f32(const oracle_pbr *p, int64_t *indptr, int64_t *indices, float *data);
int oracle_pbr_to_csr_f64(const oracle_pbr *p, int64_t *indptr, int64_t *indices, double *data);

#ifdef __cplusplus
}
#endif
#endif
