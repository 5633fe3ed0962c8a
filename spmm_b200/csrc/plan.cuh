// plan.cuh -- layout of a BOO product plan (spmm_boo_plan_build): a
// caller-owned device buffer of per-matrix tables the product reads instead
// of recomputing them on every call.  The layout follows from the matrix's
// size fields alone, so building and using a plan agree without reading the
// buffer on the host.
#pragma once

#include "common.cuh"

namespace spmm {

struct PlanLayout {
    size_t rg_blk;      // int32[n_rg + 1]: first block of each row group (blocks sorted by group)
    size_t rv_ptr;      // row view (row_view only): int32[rows + 1] row pointers,
    size_t rv_col;      //   int32[entries] columns,
    size_t rv_val;      //   scalar[entries] values: every stored entry, rows ordered by (column, value)
    size_t total;
    bool row_view;
    int64_t entries;
};

inline size_t plan_align(size_t v) { return (v + 255) & ~(size_t)255; }

// Remainder-major matrices (remainder >= half of the nonzeros) whose blocks
// and tail still hold a noticeable share (>= 1/64) of the entries -- HEM
// groups on a power-law graph -- are multiplied through a row-ordered copy of
// all their entries: one load-balanced pass then computes Y, where the block
// kernel in add mode would walk scattered blocks group by group.
inline bool plan_row_view(const spmm_boo_dev *A) {
    const int64_t entries = A->nnz_c + A->rem_nnz + A->tail_nnz;
    const bool rem_major = A->rem_nnz > 0 && 2 * A->rem_nnz >= A->total_nnz;
    return rem_major && 64 * (A->nnz_c + A->tail_nnz) >= entries && entries <= 0x7fffffffLL &&
           A->rows <= 0x7fffffffLL;
}

inline PlanLayout plan_layout(const spmm_boo_dev *A) {
    PlanLayout L{};
    const size_t sb = A->scalar_type == SPMM_F64 ? 8 : 4;
    L.entries = A->nnz_c + A->rem_nnz + A->tail_nnz;
    L.row_view = plan_row_view(A);
    size_t off = 0;
    L.rg_blk = off;
    off += plan_align(4 * (size_t)(A->n_rg + 1));
    if (L.row_view) {
        L.rv_ptr = off;
        off += plan_align(4 * (size_t)(A->rows + 1));
        L.rv_col = off;
        off += plan_align(4 * (size_t)L.entries);
        L.rv_val = off;
        off += plan_align(sb * (size_t)L.entries);
    }
    L.total = off;
    return L;
}

}  // namespace spmm
