/*
 * Scalar-generic body of the oracle, included twice by spmm_oracle.c with
 * SCALAR = float / double and SFX = f32 / f64.  Test infrastructure only.
 */

#define CAT_(a, b) a##_##b
#define CAT(a, b) CAT_(a, b)
#define FN(name) CAT(name, SFX)

/* (column, value) pair ordered like std::pair<index_t, scalar_t>::operator<,
 * the comparison the reference sorts remainder rows with
 * (boo_matrix.cpp:255, pbr_matrix.cpp:428). */
typedef struct {
    int64_t col;
    SCALAR val;
} FN(colval);

static int FN(colval_cmp)(const void *pa, const void *pb) {
    const FN(colval) *a = (const FN(colval) *)pa;
    const FN(colval) *b = (const FN(colval) *)pb;
    if (a->col < b->col) return -1;
    if (b->col < a->col) return 1;
    if (a->val < b->val) return -1;
    if (b->val < a->val) return 1;
    return 0;
}

/* Per-row bins collapsed to CSR after sorting each row by (col, value):
 * boo_matrix.cpp:249-261 and pbr_matrix.cpp:425-439. */
static int FN(collapse_bins)(int64_t rows, const int64_t *bin_ptr, FN(colval) *entries,
                             int64_t **indptr_out, int64_t **col_out, SCALAR **val_out) {
    int64_t total = bin_ptr[rows];
    int64_t *indptr = (int64_t *)malloc(sizeof(int64_t) * (size_t)(rows + 1));
    int64_t *cols = (int64_t *)malloc(sizeof(int64_t) * (size_t)(total ? total : 1));
    SCALAR *vals = (SCALAR *)malloc(sizeof(SCALAR) * (size_t)(total ? total : 1));
    if (!indptr || !cols || !vals) {
        free(indptr); free(cols); free(vals);
        return ORACLE_ENOMEM;
    }
    indptr[0] = 0;
    for (int64_t r = 0; r < rows; ++r) {
        int64_t b = bin_ptr[r], e = bin_ptr[r + 1];
        if (e - b > 1) qsort(entries + b, (size_t)(e - b), sizeof(FN(colval)), FN(colval_cmp));
        for (int64_t k = b; k < e; ++k) {
            cols[k] = entries[k].col;
            vals[k] = entries[k].val;
        }
        indptr[r + 1] = e;
    }
    *indptr_out = indptr;
    *col_out = cols;
    *val_out = vals;
    return ORACLE_OK;
}

/* ------------------------------------------------------------------------ */
/* BOO build: boo_matrix.cpp:53-274                                         */
/* ------------------------------------------------------------------------ */
int FN(oracle_csr_to_boo)(int64_t rows, int64_t cols, int64_t nnz, const int64_t *indptr,
                          const int64_t *indices, const SCALAR *data, const int32_t *row_labels,
                          int64_t n_row_labels, const int32_t *col_labels, int64_t n_col_labels,
                          int policy, int64_t threshold, int nz_order, oracle_boo *out) {
    memset(out, 0, sizeof(*out));
    /* argument checks in the reference's order (:65-94) */
    if (policy == BOO_POLICY_MERGE) return ORACLE_EMERGE;
    if (policy != BOO_POLICY_KEEP && policy != BOO_POLICY_REMAINDER &&
        policy != BOO_POLICY_TAIL) return ORACLE_EPOLICY;
    if (nz_order != BOO_ORDER_ROW && nz_order != BOO_ORDER_COL) return ORACLE_EORDER;
    if (n_row_labels != rows || n_col_labels != cols) return ORACLE_ELABELLEN;

    int64_t n_rg = 0, n_cg = 0;
    for (int64_t r = 0; r < rows; ++r) if ((int64_t)row_labels[r] + 1 > n_rg) n_rg = (int64_t)row_labels[r] + 1;
    for (int64_t c = 0; c < cols; ++c) if ((int64_t)col_labels[c] + 1 > n_cg) n_cg = (int64_t)col_labels[c] + 1;

    int64_t *row_grp_ptr, *row_ids, *row_pos, *col_grp_ptr, *col_ids, *col_pos;
    int rc = build_groups(row_labels, rows, n_rg, &row_grp_ptr, &row_ids, &row_pos);
    if (rc) return rc;
    rc = build_groups(col_labels, cols, n_cg, &col_grp_ptr, &col_ids, &col_pos);
    if (rc) { free(row_grp_ptr); free(row_ids); free(row_pos); return rc; }

    /* pass 1 (:107-125): the (row group, col group) key of every nonzero; the
     * distinct keys in ascending order are the candidate blocks. */
    int64_t *keys = (int64_t *)calloc((size_t)(nnz ? nnz : 1), sizeof(int64_t));
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = indptr[r]; j < indptr[r + 1]; ++j)
            keys[j] = (int64_t)row_labels[r] * n_cg + (int64_t)col_labels[indices[j]];
    int64_t *ukeys = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nnz ? nnz : 1));
    memcpy(ukeys, keys, sizeof(int64_t) * (size_t)nnz);
    qsort(ukeys, (size_t)nnz, sizeof(int64_t), cmp_i64);
    int64_t n_keys = 0;
    int64_t *ucount = (int64_t *)calloc((size_t)(nnz ? nnz : 1), sizeof(int64_t));
    for (int64_t i = 0; i < nnz; ++i) {
        if (n_keys == 0 || ukeys[n_keys - 1] != ukeys[i]) ukeys[n_keys++] = ukeys[i];
        ucount[n_keys - 1]++;
    }

    /* block selection (:127-171) */
    const int spills = (policy == BOO_POLICY_REMAINDER || policy == BOO_POLICY_TAIL);
    int64_t *key_block = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_keys ? n_keys : 1));
    int64_t *blk_row_grp = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_keys ? n_keys : 1));
    int64_t *blk_col_grp = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_keys ? n_keys : 1));
    int64_t *blk_nz_ptr = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_keys + 1));
    uint8_t *blk_shift = (uint8_t *)malloc((size_t)(n_keys ? n_keys : 1));
    int64_t nb = 0, running = 0, max_nr = 0, max_nc = 0, max_nnz_blk = 0;
    blk_nz_ptr[0] = 0;
    rc = ORACLE_OK;
    for (int64_t u = 0; u < n_keys; ++u) {
        key_block[u] = -1;
        int64_t cnt = ucount[u];
        if (spills && cnt < threshold) continue;
        int64_t rg = ukeys[u] / n_cg, cg = ukeys[u] % n_cg;
        int64_t n_r = row_grp_ptr[rg + 1] - row_grp_ptr[rg];
        int64_t n_c = col_grp_ptr[cg + 1] - col_grp_ptr[cg];
        uint8_t shift = ceil_log2_u32((uint32_t)n_c);
        uint64_t span = ((uint64_t)(n_r - 1) << shift) + (uint64_t)(n_c - 1);
        if (span > 0xFFFFull) { rc = ORACLE_EU16; break; }
        key_block[u] = nb;
        blk_row_grp[nb] = rg;
        blk_col_grp[nb] = cg;
        blk_shift[nb] = shift;
        running += cnt;
        blk_nz_ptr[nb + 1] = running;
        ++nb;
        if (n_r > max_nr) max_nr = n_r;
        if (n_c > max_nc) max_nc = n_c;
        if (cnt > max_nnz_blk) max_nnz_blk = cnt;
    }
    free(ucount);
    if (rc) {
        free(keys); free(ukeys); free(key_block); free(blk_row_grp); free(blk_col_grp);
        free(blk_nz_ptr); free(blk_shift); free(row_grp_ptr); free(row_ids); free(row_pos);
        free(col_grp_ptr); free(col_ids); free(col_pos);
        return rc;
    }

    /* pass 2 (:173-209): place every nonzero in CSR traversal order */
    uint16_t *nz_idx = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(running ? running : 1));
    SCALAR *nz_val = (SCALAR *)malloc(sizeof(SCALAR) * (size_t)(running ? running : 1));
    int64_t *cursor = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nb ? nb : 1));
    for (int64_t b = 0; b < nb; ++b) cursor[b] = blk_nz_ptr[b];
    int64_t *bin_ptr = (int64_t *)calloc((size_t)(rows + 1), sizeof(int64_t));
    int64_t n_spill = 0;
    int64_t *spill_j = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nnz ? nnz : 1));
    for (int64_t r = 0; r < rows; ++r) {
        int64_t local_row = row_pos[r];
        for (int64_t j = indptr[r]; j < indptr[r + 1]; ++j) {
            int64_t c = indices[j];
            int64_t u = find_key(ukeys, n_keys, keys[j]);
            int64_t b = key_block[u];
            if (b < 0) {
                spill_j[n_spill++] = j;
                bin_ptr[r + 1]++;
                continue;
            }
            int64_t slot = cursor[b]++;
            nz_idx[slot] = (uint16_t)(((uint32_t)local_row << blk_shift[b]) | (uint32_t)col_pos[c]);
            nz_val[slot] = data[j];
        }
    }
    free(cursor);
    free(key_block);
    free(ukeys);
    free(keys);

    /* in-block ordering (:211-247): sort by (key, original slot) */
    {
        uint64_t *tmp = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(max_nnz_blk ? max_nnz_blk : 1));
        uint16_t *idx_tmp = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(max_nnz_blk ? max_nnz_blk : 1));
        SCALAR *val_tmp = (SCALAR *)malloc(sizeof(SCALAR) * (size_t)(max_nnz_blk ? max_nnz_blk : 1));
        for (int64_t b = 0; b < nb; ++b) {
            int64_t beg = blk_nz_ptr[b], end = blk_nz_ptr[b + 1];
            if (end - beg < 2) continue;
            uint32_t shift = blk_shift[b];
            uint32_t mask = (1u << shift) - 1u;
            for (int64_t k = beg; k < end; ++k) {
                uint32_t idx = nz_idx[k];
                uint32_t key = (nz_order == BOO_ORDER_ROW) ? idx : (((idx & mask) << 16) | (idx >> shift));
                /* key in the high word, slot (unique) in the low word */
                tmp[k - beg] = ((uint64_t)key << 32) | (uint64_t)(uint32_t)k;
            }
            qsort(tmp, (size_t)(end - beg), sizeof(uint64_t), cmp_u64);
            for (int64_t t = 0; t < end - beg; ++t) {
                int64_t src = (int64_t)(uint32_t)(tmp[t] & 0xFFFFFFFFull);
                idx_tmp[t] = nz_idx[src];
                val_tmp[t] = nz_val[src];
            }
            memcpy(nz_idx + beg, idx_tmp, sizeof(uint16_t) * (size_t)(end - beg));
            memcpy(nz_val + beg, val_tmp, sizeof(SCALAR) * (size_t)(end - beg));
        }
        free(tmp); free(idx_tmp); free(val_tmp);
    }

    /* spilled nonzeros: flat COO tail in CSR traversal order (:194-198), or
     * per-row remainder bins sorted by (col, value) (:249-261) */
    int64_t *rem_indptr = NULL, *rem_col = NULL, *tail_row = NULL, *tail_col = NULL;
    SCALAR *rem_vals = NULL, *tail_val = NULL;
    int64_t rem_nnz = 0, tail_nnz = 0;
    if (policy == BOO_POLICY_TAIL) {
        tail_nnz = n_spill;
        tail_row = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_spill ? n_spill : 1));
        tail_col = (int64_t *)malloc(sizeof(int64_t) * (size_t)(n_spill ? n_spill : 1));
        tail_val = (SCALAR *)malloc(sizeof(SCALAR) * (size_t)(n_spill ? n_spill : 1));
        int64_t t = 0;
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t q = 0; q < bin_ptr[r + 1]; ++q, ++t) {
                tail_row[t] = r;
                tail_col[t] = indices[spill_j[t]];
                tail_val[t] = data[spill_j[t]];
            }
        memset(bin_ptr, 0, sizeof(int64_t) * (size_t)(rows + 1));
        rem_indptr = (int64_t *)calloc((size_t)(rows + 1), sizeof(int64_t));
        rem_col = (int64_t *)malloc(sizeof(int64_t));
        rem_vals = (SCALAR *)malloc(sizeof(SCALAR));
    } else {
        for (int64_t r = 0; r < rows; ++r) bin_ptr[r + 1] += bin_ptr[r];
        FN(colval) *entries = (FN(colval) *)malloc(sizeof(FN(colval)) * (size_t)(n_spill ? n_spill : 1));
        for (int64_t t = 0; t < n_spill; ++t) {
            entries[t].col = indices[spill_j[t]];
            entries[t].val = data[spill_j[t]];
        }
        rc = FN(collapse_bins)(rows, bin_ptr, entries, &rem_indptr, &rem_col, &rem_vals);
        free(entries);
        rem_nnz = n_spill;
        tail_row = (int64_t *)malloc(sizeof(int64_t));
        tail_col = (int64_t *)malloc(sizeof(int64_t));
        tail_val = (SCALAR *)malloc(sizeof(SCALAR));
    }
    free(bin_ptr);
    free(spill_j);
    free(row_pos);
    free(col_pos);

    out->rows = rows; out->cols = cols; out->total_nnz = nnz;
    out->n_rg = n_rg; out->n_cg = n_cg; out->nb = nb; out->nnz_c = running;
    out->rem_nnz = rem_nnz; out->tail_nnz = tail_nnz;
    out->max_nr = max_nr; out->max_nc = max_nc; out->max_nnz_blk = max_nnz_blk;
    out->nz_order = nz_order; out->scalar_size = (int32_t)sizeof(SCALAR);
    out->row_grp_ptr = row_grp_ptr; out->row_ids = row_ids;
    out->col_grp_ptr = col_grp_ptr; out->col_ids = col_ids;
    out->blk_row_grp = blk_row_grp; out->blk_col_grp = blk_col_grp;
    out->blk_nz_ptr = blk_nz_ptr; out->blk_shift = blk_shift;
    out->nz_idx = nz_idx; out->nz_val = nz_val;
    out->rem_indptr = rem_indptr; out->rem_col_ind = rem_col; out->rem_vals = rem_vals;
    out->tail_row = tail_row; out->tail_col = tail_col; out->tail_val = tail_val;
    return rc;
}

/* ------------------------------------------------------------------------ */
/* BOO CPU SpMM: boo_matrix.cpp:336-396 (blocks, then remainder, then tail)  */
/* ------------------------------------------------------------------------ */
void FN(oracle_boo_matmul)(int64_t rows, int64_t cols, int64_t nb, const int64_t *row_grp_ptr,
                           const int64_t *row_ids, const int64_t *col_grp_ptr,
                           const int64_t *col_ids, const int64_t *blk_row_grp,
                           const int64_t *blk_col_grp, const int64_t *blk_nz_ptr,
                           const uint8_t *blk_shift, const uint16_t *nz_idx, const SCALAR *nz_val,
                           const int64_t *rem_indptr, const int64_t *rem_col_ind,
                           const SCALAR *rem_vals, int64_t tail_nnz, const int64_t *tail_row,
                           const int64_t *tail_col, const SCALAR *tail_val, const SCALAR *x,
                           int64_t batch, int64_t K, SCALAR *y) {
    memset(y, 0, sizeof(SCALAR) * (size_t)(batch * rows * K));
    for (int64_t bt = 0; bt < batch; ++bt) {
        const SCALAR *xb = x + bt * cols * K;
        SCALAR *yb = y + bt * rows * K;
        for (int64_t b = 0; b < nb; ++b) {
            int64_t rbase = row_grp_ptr[blk_row_grp[b]];
            int64_t cbase = col_grp_ptr[blk_col_grp[b]];
            uint32_t shift = blk_shift[b];
            uint32_t mask = (1u << shift) - 1u;
            for (int64_t k = blk_nz_ptr[b]; k < blk_nz_ptr[b + 1]; ++k) {
                uint32_t idx = nz_idx[k];
                int64_t gr = row_ids[rbase + (idx >> shift)];
                int64_t gc = col_ids[cbase + (idx & mask)];
                SCALAR v = nz_val[k];
                const SCALAR *xr = xb + gc * K;
                SCALAR *yr = yb + gr * K;
                for (int64_t f = 0; f < K; ++f) yr[f] += v * xr[f];
            }
        }
        for (int64_t r = 0; r < rows; ++r) {
            SCALAR *yr = yb + r * K;
            for (int64_t j = rem_indptr[r]; j < rem_indptr[r + 1]; ++j) {
                SCALAR v = rem_vals[j];
                const SCALAR *xr = xb + rem_col_ind[j] * K;
                for (int64_t f = 0; f < K; ++f) yr[f] += v * xr[f];
            }
        }
        for (int64_t k = 0; k < tail_nnz; ++k) {
            SCALAR v = tail_val[k];
            const SCALAR *xr = xb + tail_col[k] * K;
            SCALAR *yr = yb + tail_row[k] * K;
            for (int64_t f = 0; f < K; ++f) yr[f] += v * xr[f];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* BOO -> CSR: boo_matrix.cpp:277-333                                        */
/* ------------------------------------------------------------------------ */
void FN(oracle_boo_to_csr)(const oracle_boo *bm, int64_t *indptr, int64_t *indices, SCALAR *data) {
    int64_t rows = bm->rows;
    int64_t *cnt = (int64_t *)calloc((size_t)(rows + 1), sizeof(int64_t));
    const SCALAR *nz_val = (const SCALAR *)bm->nz_val;
    const SCALAR *rem_vals = (const SCALAR *)bm->rem_vals;
    const SCALAR *tail_val = (const SCALAR *)bm->tail_val;
    for (int64_t b = 0; b < bm->nb; ++b) {
        int64_t rbase = bm->row_grp_ptr[bm->blk_row_grp[b]];
        uint32_t shift = bm->blk_shift[b];
        for (int64_t k = bm->blk_nz_ptr[b]; k < bm->blk_nz_ptr[b + 1]; ++k)
            cnt[bm->row_ids[rbase + (bm->nz_idx[k] >> shift)] + 1]++;
    }
    for (int64_t r = 0; r < rows; ++r) cnt[r + 1] += bm->rem_indptr[r + 1] - bm->rem_indptr[r];
    for (int64_t k = 0; k < bm->tail_nnz; ++k) cnt[bm->tail_row[k] + 1]++;
    for (int64_t r = 0; r < rows; ++r) cnt[r + 1] += cnt[r];
    int64_t total = cnt[rows];
    FN(colval) *e = (FN(colval) *)malloc(sizeof(FN(colval)) * (size_t)(total ? total : 1));
    int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * (size_t)(rows ? rows : 1));
    for (int64_t r = 0; r < rows; ++r) cur[r] = cnt[r];
    /* same bin-fill order as the reference: blocks, remainder, tail */
    for (int64_t b = 0; b < bm->nb; ++b) {
        int64_t rbase = bm->row_grp_ptr[bm->blk_row_grp[b]];
        int64_t cbase = bm->col_grp_ptr[bm->blk_col_grp[b]];
        uint32_t shift = bm->blk_shift[b];
        uint32_t mask = (1u << shift) - 1u;
        for (int64_t k = bm->blk_nz_ptr[b]; k < bm->blk_nz_ptr[b + 1]; ++k) {
            uint32_t idx = bm->nz_idx[k];
            int64_t gr = bm->row_ids[rbase + (idx >> shift)];
            FN(colval) *slot = &e[cur[gr]++];
            slot->col = bm->col_ids[cbase + (idx & mask)];
            slot->val = nz_val[k];
        }
    }
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = bm->rem_indptr[r]; j < bm->rem_indptr[r + 1]; ++j) {
            FN(colval) *slot = &e[cur[r]++];
            slot->col = bm->rem_col_ind[j];
            slot->val = rem_vals[j];
        }
    for (int64_t k = 0; k < bm->tail_nnz; ++k) {
        FN(colval) *slot = &e[cur[bm->tail_row[k]]++];
        slot->col = bm->tail_col[k];
        slot->val = tail_val[k];
    }
    indptr[0] = 0;
    for (int64_t r = 0; r < rows; ++r) {
        int64_t b = cnt[r], en = cnt[r + 1];
        if (en - b > 1) qsort(e + b, (size_t)(en - b), sizeof(FN(colval)), FN(colval_cmp));
        for (int64_t k = b; k < en; ++k) { indices[k] = e[k].col; data[k] = e[k].val; }
        indptr[r + 1] = en;
    }
    free(e); free(cur); free(cnt);
}

/* ------------------------------------------------------------------------ */
/* PBR build: pbr_matrix.cpp:333-448, canonical block order                  */
/* ------------------------------------------------------------------------ */
int FN(oracle_csr_to_pbr)(int64_t rows, int64_t cols, int64_t nnz, const int64_t *indptr,
                          const int64_t *indices, const SCALAR *data, int64_t br, int64_t bc,
                          uint8_t min_nnz_per_block, oracle_pbr *out) {
    memset(out, 0, sizeof(*out));
    const int64_t n_bcol = (cols + bc - 1) / bc;
    /* one record per nonzero: block key, bit, CSR position; sorted by (key, j)
     * so each block's values keep CSR traversal order (:389). */
    typedef struct { int64_t key; int64_t j; int64_t bit; } rec_t;
    rec_t *rec = (rec_t *)malloc(sizeof(rec_t) * (size_t)(nnz ? nnz : 1));
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = indptr[r]; j < indptr[r + 1]; ++j) {
            int64_t c = indices[j];
            rec[j].key = (r / br) * n_bcol + c / bc;
            rec[j].j = j;
            rec[j].bit = (r % br) * bc + c % bc;
        }
    qsort(rec, (size_t)nnz, sizeof(rec_t), cmp_rec3);

    /* worst case: every nonzero its own block */
    uint64_t *codes = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(nnz ? nnz : 1));
    int64_t *coords = (int64_t *)malloc(sizeof(int64_t) * (size_t)(2 * (nnz ? nnz : 1)));
    int64_t *offsets = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nnz + 1));
    SCALAR *bdata = (SCALAR *)malloc(sizeof(SCALAR) * (size_t)(nnz ? nnz : 1));
    int64_t *bin_cnt = (int64_t *)calloc((size_t)(rows + 1), sizeof(int64_t));
    FN(colval) *spill = (FN(colval) *)malloc(sizeof(FN(colval)) * (size_t)(nnz ? nnz : 1));
    int64_t *spill_row = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nnz ? nnz : 1));
    int64_t nb = 0, nnz_c = 0, n_spill = 0, cur_off = 0;
    offsets[0] = 0;
    for (int64_t s = 0; s < nnz;) {
        int64_t e = s;
        uint64_t code = 0;
        while (e < nnz && rec[e].key == rec[s].key) { code |= 1ull << rec[e].bit; ++e; }
        int64_t stripe = rec[s].key / n_bcol, bcol = rec[s].key % n_bcol;
        int64_t row0 = stripe * br, col0 = bcol * bc;
        int pc = __builtin_popcountll(code);
        if (pc >= (int)min_nnz_per_block) {
            /* kept (:398-406): all values appended, offset advances by popcount */
            codes[nb] = code;
            coords[2 * nb] = row0;
            coords[2 * nb + 1] = col0;
            for (int64_t t = s; t < e; ++t) bdata[nnz_c++] = data[rec[t].j];
            cur_off += pc;
            offsets[++nb] = cur_off;
        } else {
            /* spilled (:407-416): k-th set bit in bit order takes the k-th value
             * in traversal order */
            int64_t k = 0;
            for (int64_t ro = 0; ro < br; ++ro)
                for (int64_t co = 0; co < bc; ++co)
                    if (code >> (ro * bc + co) & 1ull) {
                        spill_row[n_spill] = row0 + ro;
                        spill[n_spill].col = col0 + co;
                        spill[n_spill].val = data[rec[s + k].j];
                        bin_cnt[row0 + ro + 1]++;
                        ++n_spill;
                        ++k;
                    }
        }
        s = e;
    }
    free(rec);
    for (int64_t r = 0; r < rows; ++r) bin_cnt[r + 1] += bin_cnt[r];
    FN(colval) *binned = (FN(colval) *)malloc(sizeof(FN(colval)) * (size_t)(n_spill ? n_spill : 1));
    int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * (size_t)(rows ? rows : 1));
    for (int64_t r = 0; r < rows; ++r) cur[r] = bin_cnt[r];
    for (int64_t t = 0; t < n_spill; ++t) binned[cur[spill_row[t]]++] = spill[t];
    free(cur); free(spill); free(spill_row);
    int64_t *rem_indptr, *rem_col;
    SCALAR *rem_vals;
    int rc = FN(collapse_bins)(rows, bin_cnt, binned, &rem_indptr, &rem_col, &rem_vals);
    free(binned); free(bin_cnt);
    out->rows = rows; out->cols = cols; out->block_rows = br; out->block_cols = bc;
    out->total_nnz = nnz; out->nb = nb; out->nnz_c = nnz_c; out->rem_nnz = n_spill;
    out->scalar_size = (int32_t)sizeof(SCALAR);
    out->codes = codes; out->coords = coords; out->offsets = offsets; out->data = bdata;
    out->rem_indptr = rem_indptr; out->rem_col_ind = rem_col; out->rem_vals = rem_vals;
    return rc;
}

/* ------------------------------------------------------------------------ */
/* PBR CPU SpMM: pbr_matrix.cpp:17-68                                        */
/* ------------------------------------------------------------------------ */
void FN(oracle_pbr_matmul)(int64_t rows, int64_t cols, int64_t br, int64_t bc, int64_t nb,
                           const uint64_t *codes, const int64_t *coords, const SCALAR *data,
                           const int64_t *rem_indptr, const int64_t *rem_col_ind,
                           const SCALAR *rem_vals, const SCALAR *x, int64_t batch, int64_t K,
                           SCALAR *y) {
    memset(y, 0, sizeof(SCALAR) * (size_t)(batch * rows * K));
    for (int64_t bt = 0; bt < batch; ++bt) {
        const SCALAR *xb = x + bt * cols * K;
        SCALAR *yb = y + bt * rows * K;
        int64_t di = 0;
        for (int64_t b = 0; b < nb; ++b) {
            uint64_t code = codes[b];
            for (int64_t r = 0; r < br; ++r) {
                int64_t gr = coords[2 * b] + r;
                if (gr >= rows) continue;
                for (int64_t c = 0; c < bc; ++c) {
                    int64_t gc = coords[2 * b + 1] + c;
                    if (gc >= cols) continue;
                    if (code >> (r * bc + c) & 1ull) {
                        SCALAR v = data[di++];
                        for (int64_t f = 0; f < K; ++f) yb[gr * K + f] += v * xb[gc * K + f];
                    }
                }
            }
        }
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t j = rem_indptr[r]; j < rem_indptr[r + 1]; ++j) {
                SCALAR v = rem_vals[j];
                int64_t c = rem_col_ind[j];
                for (int64_t f = 0; f < K; ++f) yb[r * K + f] += v * xb[c * K + f];
            }
    }
}

/* ------------------------------------------------------------------------ */
/* PBR -> CSR: pbr_matrix.cpp:279-331                                        */
/* ------------------------------------------------------------------------ */
int FN(oracle_pbr_to_csr)(const oracle_pbr *p, int64_t *indptr, int64_t *indices, SCALAR *data) {
    int64_t rows = p->rows;
    const SCALAR *bdata = (const SCALAR *)p->data;
    const SCALAR *rvals = (const SCALAR *)p->rem_vals;
    int64_t *cnt = (int64_t *)calloc((size_t)(rows + 1), sizeof(int64_t));
    for (int64_t b = 0; b < p->nb; ++b)
        for (int64_t r = 0; r < p->block_rows; ++r)
            for (int64_t c = 0; c < p->block_cols; ++c)
                if (p->codes[b] >> (r * p->block_cols + c) & 1ull) {
                    if (p->coords[2 * b] + r >= rows) { free(cnt); return 1; }
                    if (p->coords[2 * b + 1] + c >= p->cols) continue;
                    cnt[p->coords[2 * b] + r + 1]++;
                }
    for (int64_t r = 0; r < rows; ++r) cnt[r + 1] += cnt[r] + (p->rem_indptr[r + 1] - p->rem_indptr[r]);
    int64_t total = cnt[rows];
    FN(colval) *e = (FN(colval) *)malloc(sizeof(FN(colval)) * (size_t)(total ? total : 1));
    int64_t *cur = (int64_t *)malloc(sizeof(int64_t) * (size_t)(rows ? rows : 1));
    for (int64_t r = 0; r < rows; ++r) cur[r] = cnt[r];
    int64_t di = 0;
    for (int64_t b = 0; b < p->nb; ++b)
        for (int64_t r = 0; r < p->block_rows; ++r)
            for (int64_t c = 0; c < p->block_cols; ++c) {
                if (p->coords[2 * b + 1] + c >= p->cols) continue;
                if (p->codes[b] >> (r * p->block_cols + c) & 1ull) {
                    int64_t gr = p->coords[2 * b] + r;
                    e[cur[gr]].col = p->coords[2 * b + 1] + c;
                    e[cur[gr]++].val = bdata[di++];
                }
            }
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = p->rem_indptr[r]; j < p->rem_indptr[r + 1]; ++j) {
            e[cur[r]].col = p->rem_col_ind[j];
            e[cur[r]++].val = rvals[j];
        }
    indptr[0] = 0;
    for (int64_t r = 0; r < rows; ++r) {
        int64_t b = cnt[r], en = cnt[r + 1];
        if (en - b > 1) qsort(e + b, (size_t)(en - b), sizeof(FN(colval)), FN(colval_cmp));
        for (int64_t k = b; k < en; ++k) { indices[k] = e[k].col; data[k] = e[k].val; }
        indptr[r + 1] = en;
    }
    free(e); free(cur); free(cnt);
    return 0;
}

#undef FN
#undef CAT
#undef CAT_
