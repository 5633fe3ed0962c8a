/*
 * spmm_oracle.c -- CPU restatement of the reference's BOO/PBR builders and CPU
 * SpMM.  TEST INFRASTRUCTURE ONLY: see spmm_oracle.h for what pins it and for
 * the documented limits.  Citations are to files of the reference project
 * (torch_fast_spdmm/boo_matrix/boo_matrix.cpp, torch_fast_spdmm/pbr_matrix/
 * pbr_matrix.cpp).
 */
#include "spmm_oracle.h"

#include <stdlib.h>
#include <string.h>

/* boo_small_block_policy_t / boo_nz_order_t values (boo_matrix.hpp:41-55) */
#define BOO_POLICY_KEEP 0
#define BOO_POLICY_MERGE 1
#define BOO_POLICY_REMAINDER 2
#define BOO_POLICY_TAIL 3
#define BOO_ORDER_ROW 0
#define BOO_ORDER_COL 1

/* ceil(log2(v)); 1 -> 0 (boo_matrix.cpp:12-16) */
static uint8_t ceil_log2_u32(uint32_t v) {
    uint8_t s = 0;
    while ((1u << s) < v) ++s;
    return s;
}

static int cmp_i64(const void *a, const void *b) {
    int64_t x = *(const int64_t *)a, y = *(const int64_t *)b;
    return (x > y) - (x < y);
}

static int cmp_u64(const void *a, const void *b) {
    uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return (x > y) - (x < y);
}

/* records sorted by (key, j) */
static int cmp_rec3(const void *a, const void *b) {
    const int64_t *x = (const int64_t *)a, *y = (const int64_t *)b;
    if (x[0] != y[0]) return (x[0] > y[0]) - (x[0] < y[0]);
    return (x[1] > y[1]) - (x[1] < y[1]);
}

/* index of `key` in the ascending unique array `ukeys` (key is present) */
static int64_t find_key(const int64_t *ukeys, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (hi - lo > 1) {
        int64_t mid = lo + (hi - lo) / 2;
        if (ukeys[mid] <= key) lo = mid; else hi = mid;
    }
    return lo;
}

/* Counting sort of labels into groups (boo_matrix.cpp:18-48): group_ptr is
 * the exclusive scan of the label histogram, ids ascending within a group,
 * pos[i] = local index of i inside its group. */
static int build_groups(const int32_t *labels, int64_t n, int64_t n_groups, int64_t **group_ptr_out,
                        int64_t **ids_out, int64_t **pos_out) {
    int64_t *gp = (int64_t *)calloc((size_t)(n_groups + 1), sizeof(int64_t));
    int64_t *ids = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n ? n : 1));
    int64_t *pos = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n ? n : 1));
    int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_groups ? n_groups : 1));
    if (!gp || !ids || !pos || !cur) {
        free(gp); free(ids); free(pos); free(cur);
        return ORACLE_ENOMEM;
    }
    for (int64_t i = 0; i < n; ++i) {
        int32_t l = labels[i];
        if (l < 0 || (int64_t)l >= n_groups) {
            free(gp); free(ids); free(pos); free(cur);
            return ORACLE_ELABEL;
        }
        gp[l + 1]++;
    }
    for (int64_t g = 0; g < n_groups; ++g) gp[g + 1] += gp[g];
    for (int64_t g = 0; g < n_groups; ++g) cur[g] = gp[g];
    for (int64_t i = 0; i < n; ++i) {
        int64_t slot = cur[labels[i]]++;
        ids[slot] = i;
        pos[i] = slot - gp[labels[i]];
    }
    free(cur);
    *group_ptr_out = gp;
    *ids_out = ids;
    *pos_out = pos;
    return ORACLE_OK;
}

#define SCALAR float
#define SFX f32
#include "spmm_oracle_body.h"
#undef SCALAR
#undef SFX

#define SCALAR double
#define SFX f64
#include "spmm_oracle_body.h"
#undef SCALAR
#undef SFX

void oracle_boo_free(oracle_boo *b) {
    free(b->row_grp_ptr); free(b->row_ids); free(b->col_grp_ptr); free(b->col_ids);
    free(b->blk_row_grp); free(b->blk_col_grp); free(b->blk_nz_ptr); free(b->blk_shift);
    free(b->nz_idx); free(b->nz_val); free(b->rem_indptr); free(b->rem_col_ind);
    free(b->rem_vals); free(b->tail_row); free(b->tail_col); free(b->tail_val);
    memset(b, 0, sizeof(*b));
}

void oracle_pbr_free(oracle_pbr *p) {
    free(p->codes); free(p->coords); free(p->offsets); free(p->data);
    free(p->rem_indptr); free(p->rem_col_ind); free(p->rem_vals);
    memset(p, 0, sizeof(*p));
}
