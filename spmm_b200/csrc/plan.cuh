// plan.cuh -- layout of a BOO product plan (spmm_boo_plan_build): a
// caller-owned device buffer of per-matrix tables the product reads instead
// of recomputing them on every call.  The layout follows from the matrix's
// size fields alone, so building and using a plan agree without reading the
// buffer on the host.
#pragma once

#include "common.cuh"

namespace spmm {

// Blocks with at least kDenseNnz nonzeros go through the tensor cores as
// dense tiles of their own (shared by the product and the plan builder).
constexpr int kDenseNnz = 48;

struct PlanLayout {
    size_t rg_blk;      // int32[n_rg + 1]: first block of each row group (blocks sorted by group)
    size_t packed;      // tensor-core matrices (packing): uint8[nb], 1 = the block's entries go
                        //   through a packed tensor-core tile, not the CUDA cores;
    size_t rg_slot;     //   int32[n_rg + 1]: first packed slot of each row group;
    size_t slots;       //   int32[2 nb]: packed slots, block * 16 + quad (4 columns of its group)
    size_t cg_ident;    //   int32, 1 when col_ids[k] == k for every k (column groups are runs of
                        //   consecutive X rows: 64-column panels are read straight from X)
    bool packing;
    int pw;             //   panel width of the tensor-core product (32 or 64 columns)
    size_t rv_ptr;      // row view (row_view only): int32[rows + 1] row pointers,
    size_t rv_col;      //   int32[entries] columns,
    size_t rv_val;      //   scalar[entries] values: every stored entry, rows ordered by (column, value)
    size_t rv_ident;    // short_rows only: int32, 1 when row_ids[k] == k for every position k
    size_t total;
    bool row_view;
    bool short_rows;    // the row view serves a warp-per-row product (not remainder-major)
    int64_t entries;
};

inline size_t plan_align(size_t v) { return (v + 255) & ~(size_t)255; }

// Remainder-major matrices (remainder >= half of the nonzeros) whose blocks
// and tail still hold a noticeable share (>= 1/64) of the entries -- HEM
// groups on a power-law graph -- are multiplied through a row-ordered copy of
// all their entries: one load-balanced pass then computes Y, where the block
// kernel in add mode would walk scattered blocks group by group.
inline bool plan_row_view_rem(const spmm_boo_dev *A) {
    const int64_t entries = A->nnz_c + A->rem_nnz + A->tail_nnz;
    const bool rem_major = A->rem_nnz > 0 && 2 * A->rem_nnz >= A->total_nnz;
    return rem_major && 64 * (A->nnz_c + A->tail_nnz) >= entries && entries <= 0x7fffffffLL &&
           A->rows <= 0x7fffffffLL;
}

// Other matrices of at most kShortRow entries per row on average (a 2-D
// Laplacian: 5) are multiplied through the same copy a warp per row: the
// block kernel's per-group chain of dependent loads outweighs their few
// products.
constexpr int64_t kShortRow = 16;
inline bool plan_short_rows(const spmm_boo_dev *A) {
    const int64_t entries = A->nnz_c + A->rem_nnz + A->tail_nnz;
    const bool rem_major = A->rem_nnz > 0 && 2 * A->rem_nnz >= A->total_nnz;
    return !rem_major && A->rows > 0 && entries > 0 && entries <= kShortRow * A->rows &&
           entries <= 0x7fffffffLL && A->rows <= 0x7fffffffLL;
}

inline bool plan_row_view(const spmm_boo_dev *A) { return plan_row_view_rem(A) || plan_short_rows(A); }

// Matrices the tensor-core product can take (float32, groups up to 64 x 64):
// their sparse blocks whose entries lie in at most two 4-column quads are
// packed, quad by quad, into extra tensor-core tiles (plan_build).
inline bool plan_packing(const spmm_boo_dev *A) {
    return A->scalar_type == SPMM_F32 && A->nb > 0 && A->nb < (1ll << 27) && A->max_nr <= 64 &&
           A->max_nc <= 64;
}

inline PlanLayout plan_layout(const spmm_boo_dev *A) {
    PlanLayout L{};
    const size_t sb = A->scalar_type == SPMM_F64 ? 8 : 4;
    L.entries = A->nnz_c + A->rem_nnz + A->tail_nnz;
    L.row_view = plan_row_view(A);
    L.short_rows = plan_short_rows(A);
    L.packing = plan_packing(A);
    L.pw = A->max_nr <= 32 && A->max_nc <= 32 ? 32 : 64;
    size_t off = 0;
    L.rg_blk = off;
    off += plan_align(4 * (size_t)(A->n_rg + 1));
    if (L.packing) {
        L.packed = off;
        off += plan_align((size_t)A->nb);
        L.rg_slot = off;
        off += plan_align(4 * (size_t)(A->n_rg + 1));
        L.slots = off;
        off += plan_align(8 * (size_t)A->nb);
        L.cg_ident = off;
        off += plan_align(4);
    }
    if (L.row_view) {
        L.rv_ptr = off;
        off += plan_align(4 * (size_t)(A->rows + 1));
        L.rv_col = off;
        off += plan_align(4 * (size_t)L.entries);
        L.rv_val = off;
        off += plan_align(sb * (size_t)L.entries);
    }
    if (L.short_rows) {
        L.rv_ident = off;
        off += plan_align(4);
    }
    L.total = off;
    return L;
}

}  // namespace spmm
