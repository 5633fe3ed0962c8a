// build_boo.cu -- GPU construction of the BOO format from a device CSR.
//
// Reproduces the reference builder csr_to_boo (torch_fast_spdmm/boo_matrix/
// boo_matrix.cpp:53-274) array for array:
//   * groups: counting sort of the labels, ids ascending inside a group
//     (boo_matrix.cpp:23-48)               -> stable radix sort of (label, id)
//   * blocks: distinct (row group, col group) keys in ascending order
//     (:107-125)                           -> stable radix sort of the nonzeros
//     by (block key << 16 | in-block key); ties keep CSR order, which is the
//     reference's (key, slot) tie-break (:219-246)
//   * keep / spill with the uint16 span check on kept blocks (:127-171)
//   * remainder rows sorted by (col, value) (:249-261); the tail in CSR
//     traversal order (:194-198).
// Output index arrays are int32 and nz_idx uint16, the reference's GPU staging
// types (torch_fast_spdmm/torch_fast_spdmm/boo.py:71-90).
#include "build_common.cuh"

namespace spmm {
namespace {

struct BooWs {
    BuildCounters *cnt;
    int32_t *row_of;                     // nnz
    uint64_t *k0, *k1;                   // max(nnz, rows, cols)
    uint32_t *v0, *v1;
    uint32_t *sort_temp;
    int32_t *rgp, *rids, *rpos;          // rows+1, rows, rows
    int32_t *cgp, *cids, *cpos;          // cols+1, cols, cols
    uint32_t *flag;                      // nnz+1 : segment flags -> candidate block of entry
    uint32_t *bstart;                    // nnz+1 : candidate block start positions
    uint32_t *keep;                      // nnz+1 : keep flag -> kept index (scan)
    uint32_t *kcnt;                      // nnz+1 : kept counts -> compressed start (scan)
    uint32_t *spill;                     // nnz+1 : spill flag per CSR position -> position (scan)
    uint32_t *scan_temp;                 // scan temp for nnz+1 / rows+1
    int32_t *tmp_col;                    // nnz : remainder staging for the unsorted path
    double *tmp_val;                     // nnz
};

template <bool CARVE>
size_t boo_ws_layout(int64_t rows, int64_t cols, int64_t nnz, void *base, size_t cap, BooWs *ws) {
    int64_t m = nnz;
    if (rows > m) m = rows;
    if (cols > m) m = cols;
    int64_t big = nnz + 1 > rows + 1 ? nnz + 1 : rows + 1;
    if (cols + 1 > big) big = cols + 1;
    Arena a(base, cap);
    size_t used = 0;
#define CARVE_(field, T, n)                       \
    do {                                          \
        if (CARVE) ws->field = a.take<T>(n);      \
        else arena_count<T>(used, n);             \
    } while (0)
    CARVE_(cnt, BuildCounters, 1);
    CARVE_(row_of, int32_t, nnz);
    CARVE_(k0, uint64_t, m);
    CARVE_(k1, uint64_t, m);
    CARVE_(v0, uint32_t, m);
    CARVE_(v1, uint32_t, m);
    CARVE_(sort_temp, uint32_t, radix_temp_elems(m));
    CARVE_(rgp, int32_t, rows + 2);
    CARVE_(rids, int32_t, rows);
    CARVE_(rpos, int32_t, rows);
    CARVE_(cgp, int32_t, cols + 2);
    CARVE_(cids, int32_t, cols);
    CARVE_(cpos, int32_t, cols);
    CARVE_(flag, uint32_t, nnz + 1);
    CARVE_(bstart, uint32_t, nnz + 1);
    CARVE_(keep, uint32_t, nnz + 1);
    CARVE_(kcnt, uint32_t, nnz + 1);
    CARVE_(spill, uint32_t, nnz + 1);
    CARVE_(scan_temp, uint32_t, scan_temp_elems(big) + 2);
    CARVE_(tmp_col, int32_t, nnz + 1);
    CARVE_(tmp_val, double, nnz);
#undef CARVE_
    return CARVE ? a.used : used;
}

__global__ void label_max_kernel(const int32_t *__restrict__ labels, int64_t n,
                                 unsigned long long *maxp, unsigned int *err) {
    unsigned long long m = 0;
    bool bad = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int32_t l = labels[i];
        if (l < 0 || (int64_t)l >= n) bad = true;
        else if ((unsigned long long)l + 1 > m) m = (unsigned long long)l + 1;
    }
    // one atomic per warp (labels < 2^31, so the maximum fits 32 bits)
    const unsigned wm = __reduce_max_sync(kFullMask, (unsigned)m);
    const bool wbad = __any_sync(kFullMask, bad);
    if ((threadIdx.x & 31) == 0) {
        if (wbad) atomicOr(err, 1u);
        if (wm) atomicMax(maxp, (unsigned long long)wm);
    }
}

// ---- groups ---------------------------------------------------------------

__global__ void label_keys_kernel(const int32_t *__restrict__ labels, int64_t n,
                                  uint64_t *__restrict__ keys, uint32_t *__restrict__ vals,
                                  int32_t *__restrict__ hist) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int32_t l = labels[i];
        keys[i] = (uint64_t)(uint32_t)l;
        vals[i] = (uint32_t)i;
        atomicAdd(&hist[l], 1);
    }
}

// ids[s] = sorted id; pos[id] = s - group_ptr[label[id]]
__global__ void group_pos_kernel(const uint32_t *__restrict__ sorted_ids, int64_t n,
                                 const int32_t *__restrict__ labels,
                                 const int32_t *__restrict__ gptr, int32_t *__restrict__ ids,
                                 int32_t *__restrict__ pos) {
    for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n;
         s += (int64_t)gridDim.x * blockDim.x) {
        uint32_t id = sorted_ids[s];
        ids[s] = (int32_t)id;
        pos[id] = (int32_t)(s - gptr[labels[id]]);
    }
}

// key = ((rg * n_cg + cg) << 16) | in-block order key
template <typename I>
__global__ void nz_keys_kernel(const I *__restrict__ indices, const int32_t *__restrict__ row_of,
                               int64_t nnz, const int32_t *__restrict__ rl,
                               const int32_t *__restrict__ cl, const int32_t *__restrict__ rpos,
                               const int32_t *__restrict__ cpos, const int32_t *__restrict__ cgp,
                               int64_t n_cg, int nz_order, uint64_t *__restrict__ keys,
                               uint32_t *__restrict__ vals) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < nnz;
         j += (int64_t)gridDim.x * blockDim.x) {
        const int32_t r = row_of[j];
        const int32_t c = (int32_t)indices[j];
        const int32_t cg = cl[c];
        const uint32_t shift = ceil_log2_dev((uint32_t)(cgp[cg + 1] - cgp[cg]));
        const uint32_t lr = (uint32_t)rpos[r], lc = (uint32_t)cpos[c];
        uint32_t sk;
        if (nz_order == SPMM_BOO_ROWMAJOR) {
            uint64_t idx = ((uint64_t)lr << shift) | lc;
            sk = idx > 0xFFFFu ? 0xFFFFu : (uint32_t)idx;
        } else {
            // (local_col, local_row) lexicographic, packed into 16 bits; only a
            // block that fails the uint16 span check can overflow it.
            sk = (shift <= 16 && lr < (1u << (16 - shift))) ? ((lc << (16 - shift)) | lr) : 0xFFFFu;
        }
        keys[j] = (((uint64_t)rl[r] * (uint64_t)n_cg + (uint64_t)cg) << 16) | sk;
        vals[j] = (uint32_t)j;
    }
}

// ---- block discovery --------------------------------------------------------

__global__ void block_select_kernel(const uint64_t *__restrict__ keys,
                                    const uint32_t *__restrict__ bstart, uint32_t n_cand,
                                    int64_t nnz, int64_t n_cg, const int32_t *__restrict__ rgp,
                                    const int32_t *__restrict__ cgp, int spills, int64_t threshold,
                                    uint32_t *__restrict__ keep, uint32_t *__restrict__ kcnt,
                                    BuildCounters *cnt) {
    unsigned long long mr = 0, mc = 0, mn = 0;
    bool over = false;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= (int64_t)n_cand;
         b += (int64_t)gridDim.x * blockDim.x) {
        if (b == (int64_t)n_cand) { keep[b] = 0; kcnt[b] = 0; continue; }
        const uint32_t s = bstart[b];
        const uint32_t e = (b + 1 < (int64_t)n_cand) ? bstart[b + 1] : (uint32_t)nnz;
        const uint32_t count = e - s;
        const bool k = !(spills && (int64_t)count < threshold);
        keep[b] = k;
        kcnt[b] = k ? count : 0;
        if (k) {
            const uint64_t bk = keys[s] >> 16;
            const int64_t rg = (int64_t)(bk / (uint64_t)n_cg), cg = (int64_t)(bk % (uint64_t)n_cg);
            const uint32_t n_r = (uint32_t)(rgp[rg + 1] - rgp[rg]);
            const uint32_t n_c = (uint32_t)(cgp[cg + 1] - cgp[cg]);
            const uint32_t shift = ceil_log2_dev(n_c);
            const uint64_t span = ((uint64_t)(n_r - 1) << shift) + (uint64_t)(n_c - 1);
            if (span > 0xFFFFull) over = true;
            if (n_r > mr) mr = n_r;
            if (n_c > mc) mc = n_c;
            if (count > mn) mn = count;
        }
    }
    // one atomic per warp and counter (every value fits 32 bits): per-thread
    // atomics on these three words serialised the kernel at one candidate per
    // L2 atomic slot
    const unsigned wr = __reduce_max_sync(kFullMask, (unsigned)mr);
    const unsigned wc = __reduce_max_sync(kFullMask, (unsigned)mc);
    const unsigned wn = __reduce_max_sync(kFullMask, (unsigned)mn);
    const bool wover = __any_sync(kFullMask, over);
    if ((threadIdx.x & 31) == 0) {
        if (wover) atomicOr(&cnt->err_u16, 1u);
        if (wr) atomicMax(&cnt->max_nr, (unsigned long long)wr);
        if (wc) atomicMax(&cnt->max_nc, (unsigned long long)wc);
        if (wn) atomicMax(&cnt->max_nnz_blk, (unsigned long long)wn);
    }
}

// ---- emit -------------------------------------------------------------------

__global__ void emit_blocks_kernel(const uint64_t *__restrict__ keys,
                                   const uint32_t *__restrict__ bstart, uint32_t n_cand,
                                   const uint32_t *__restrict__ keep_flag,
                                   const uint32_t *__restrict__ keep_idx,
                                   const uint32_t *__restrict__ cstart, int64_t n_cg,
                                   const int32_t *__restrict__ cgp, uint32_t nb, uint32_t nnz_c,
                                   int32_t *__restrict__ brg, int32_t *__restrict__ bcg,
                                   int32_t *__restrict__ bptr, uint8_t *__restrict__ bshift) {
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < (int64_t)n_cand;
         b += (int64_t)gridDim.x * blockDim.x) {
        if (!keep_flag[b]) continue;
        const uint32_t kb = keep_idx[b];
        const uint64_t bk = keys[bstart[b]] >> 16;
        const int64_t cg = (int64_t)(bk % (uint64_t)n_cg);
        brg[kb] = (int32_t)(bk / (uint64_t)n_cg);
        bcg[kb] = (int32_t)cg;
        bptr[kb] = (int32_t)cstart[b];
        bshift[kb] = (uint8_t)ceil_log2_dev((uint32_t)(cgp[cg + 1] - cgp[cg]));
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) bptr[nb] = (int32_t)nnz_c;
}

// Sorted entry i -> its slot in the kept block, or a spill mark at its CSR
// position.  keep_raw holds the unscanned keep flags (saved before the scan).
template <typename I, typename S>
__global__ void emit_entries_kernel(const uint32_t *__restrict__ vals, int64_t nnz,
                                    const uint32_t *__restrict__ blk_of,
                                    const uint32_t *__restrict__ bstart,
                                    const uint32_t *__restrict__ keep_raw,
                                    const uint32_t *__restrict__ cstart,
                                    const I *__restrict__ indices, const S *__restrict__ values,
                                    const int32_t *__restrict__ row_of,
                                    const int32_t *__restrict__ rpos,
                                    const int32_t *__restrict__ cpos,
                                    const int32_t *__restrict__ cl,
                                    const int32_t *__restrict__ cgp, uint16_t *__restrict__ nz_idx,
                                    S *__restrict__ nz_val, uint32_t *__restrict__ spill) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nnz;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t b = blk_of[i];
        const uint32_t j = vals[i];
        if (keep_raw[b]) {
            const uint32_t p = cstart[b] + (uint32_t)(i - bstart[b]);
            const int32_t c = (int32_t)indices[j];
            const int32_t cg = cl[c];
            const uint32_t shift = ceil_log2_dev((uint32_t)(cgp[cg + 1] - cgp[cg]));
            nz_idx[p] = (uint16_t)(((uint32_t)rpos[row_of[j]] << shift) | (uint32_t)cpos[c]);
            nz_val[p] = values[j];
        } else {
            spill[j] = 1u;
        }
    }
}

// ---- drivers ------------------------------------------------------------------

struct BooArgs {
    const spmm_csr_dev *A;
    const int32_t *rl, *cl;
    int policy;
    int64_t threshold;
    int order;
};

int validate_args(const BooArgs &a) {
    SPMM_TRY(validate_csr(a.A));
    if (a.policy == SPMM_BOO_MERGE) return SPMM_EINVAL;
    if (a.policy != SPMM_BOO_KEEP && a.policy != SPMM_BOO_REMAINDER &&
        a.policy != SPMM_BOO_TAIL_BATCH)
        return SPMM_EINVAL;
    if (a.order != SPMM_BOO_ROWMAJOR && a.order != SPMM_BOO_COLMAJOR) return SPMM_EINVAL;
    if ((a.A->rows && !a.rl) || (a.A->cols && !a.cl)) return SPMM_EINVAL;
    return SPMM_OK;
}

template <typename I, typename S>
int boo_analyze_impl(const BooArgs &a, BooWs &w, spmm_boo_dev *sz, cudaStream_t s) {
    const spmm_csr_dev *A = a.A;
    const int64_t rows = A->rows, cols = A->cols, nnz = A->nnz;
    const I *indptr = (const I *)A->indptr;
    const I *indices = (const I *)A->indices;
    const int T = 256;

    SPMM_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, sizeof(BuildCounters), s));
    check_indptr_kernel<I><<<grid_for(rows + 1, T), T, 0, s>>>(indptr, rows, nnz, w.cnt);
    SPMM_LAUNCH_CHECK();
    if (rows) label_max_kernel<<<grid_for(rows, T), T, 0, s>>>(a.rl, rows, &w.cnt->n_rg, &w.cnt->err_label);
    if (cols) label_max_kernel<<<grid_for(cols, T), T, 0, s>>>(a.cl, cols, &w.cnt->n_cg, &w.cnt->err_label);
    SPMM_LAUNCH_CHECK();
    BuildCounters h;
    SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    if (h.err_index) return SPMM_EINVAL;
    if (h.err_label) return SPMM_ELABEL;
    const int64_t n_rg = (int64_t)h.n_rg, n_cg = (int64_t)h.n_cg;

    // groups: rows then cols
    for (int axis = 0; axis < 2; ++axis) {
        const int64_t n = axis ? cols : rows;
        const int64_t ng = axis ? n_cg : n_rg;
        const int32_t *lab = axis ? a.cl : a.rl;
        int32_t *gp = axis ? w.cgp : w.rgp;
        int32_t *ids = axis ? w.cids : w.rids;
        int32_t *pos = axis ? w.cpos : w.rpos;
        SPMM_CUDA_TRY(cudaMemsetAsync(gp, 0, sizeof(int32_t) * (size_t)(ng + 1), s));
        if (n == 0) continue;
        label_keys_kernel<<<grid_for(n, T), T, 0, s>>>(lab, n, w.k0, w.v0, gp);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(exclusive_scan<int32_t>(gp, gp, ng + 1, (int32_t *)w.scan_temp, nullptr, s));
        bool first;
        SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(w.k0, w.v0, w.k1, w.v1, n,
                                                      bit_width_u64((uint64_t)(ng - 1)), w.sort_temp,
                                                      &first, s));
        group_pos_kernel<<<grid_for(n, T), T, 0, s>>>(first ? w.v0 : w.v1, n, lab, gp, ids, pos);
        SPMM_LAUNCH_CHECK();
    }

    uint32_t n_cand = 0, nb = 0, nnz_c = 0;
    if (nnz > 0) {
        const int64_t warps_needed = rows;
        row_of_kernel<I><<<grid_for(warps_needed * 32, T), T, 0, s>>>(indptr, indices, rows, cols,
                                                                       w.row_of, w.cnt);
        SPMM_LAUNCH_CHECK();
        SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
        SPMM_CUDA_TRY(cudaStreamSynchronize(s));
        if (h.err_index) return SPMM_EINVAL;
        const uint64_t max_block_key = (uint64_t)n_rg * (uint64_t)n_cg - 1;
        const int key_bits = bit_width_u64(max_block_key) + 16;
        if (key_bits > 64) return SPMM_EUNSUPPORTED;
        nz_keys_kernel<I><<<grid_for(nnz, T), T, 0, s>>>(indices, w.row_of, nnz, a.rl, a.cl, w.rpos,
                                                         w.cpos, w.cgp, n_cg, a.order, w.k0, w.v0);
        SPMM_LAUNCH_CHECK();
        bool first;
        SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(w.k0, w.v0, w.k1, w.v1, nnz, key_bits,
                                                      w.sort_temp, &first, s));
        if (!first) {
            // keep the sorted pairs in (k0, v0) for the emit phase
            SPMM_CUDA_TRY(cudaMemcpyAsync(w.k0, w.k1, sizeof(uint64_t) * (size_t)nnz,
                                          cudaMemcpyDeviceToDevice, s));
            SPMM_CUDA_TRY(cudaMemcpyAsync(w.v0, w.v1, sizeof(uint32_t) * (size_t)nnz,
                                          cudaMemcpyDeviceToDevice, s));
        }
        uint32_t *tot = (uint32_t *)&w.cnt->n_cand;
        seg_flag_kernel<<<grid_for(nnz + 1, T), T, 0, s>>>(w.k0, nnz, 16, w.flag);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(exclusive_scan<uint32_t>(w.flag, w.flag, nnz + 1, w.scan_temp, tot, s));
        seg_start_kernel<<<grid_for(nnz, T), T, 0, s>>>(w.k0, nnz, 16, w.flag, w.bstart);
        SPMM_LAUNCH_CHECK();
        SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
        SPMM_CUDA_TRY(cudaStreamSynchronize(s));
        n_cand = h.n_cand;
        const int spills = (a.policy == SPMM_BOO_REMAINDER || a.policy == SPMM_BOO_TAIL_BATCH);
        block_select_kernel<<<grid_for((int64_t)n_cand + 1, T), T, 0, s>>>(
            w.k0, w.bstart, n_cand, nnz, n_cg, w.rgp, w.cgp, spills, a.threshold, w.keep, w.kcnt, w.cnt);
        SPMM_LAUNCH_CHECK();
        // keep the raw flags in `spill`'s sibling: copy keep -> tmp_col (as u32) before scanning
        SPMM_CUDA_TRY(cudaMemcpyAsync(w.tmp_col, w.keep, sizeof(uint32_t) * (size_t)(n_cand + 1),
                                      cudaMemcpyDeviceToDevice, s));
        SPMM_TRY(exclusive_scan<uint32_t>(w.keep, w.keep, (int64_t)n_cand + 1, w.scan_temp,
                                          (uint32_t *)&w.cnt->nb, s));
        SPMM_TRY(exclusive_scan<uint32_t>(w.kcnt, w.kcnt, (int64_t)n_cand + 1, w.scan_temp,
                                          (uint32_t *)&w.cnt->nnz_c, s));
        SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
        SPMM_CUDA_TRY(cudaStreamSynchronize(s));
        if (h.err_u16) return SPMM_EOVERFLOW_U16;
        nb = h.nb;
        nnz_c = h.nnz_c;
    }
    const int64_t n_spill = nnz - (int64_t)nnz_c;
    sz->rows = rows;
    sz->cols = cols;
    sz->total_nnz = nnz;
    sz->n_rg = n_rg;
    sz->n_cg = n_cg;
    sz->nb = nb;
    sz->nnz_c = nnz_c;
    sz->rem_nnz = a.policy == SPMM_BOO_TAIL_BATCH ? 0 : n_spill;
    sz->tail_nnz = a.policy == SPMM_BOO_TAIL_BATCH ? n_spill : 0;
    sz->max_nr = (int64_t)h.max_nr;
    sz->max_nc = (int64_t)h.max_nc;
    sz->max_nnz_blk = (int64_t)h.max_nnz_blk;
    sz->nz_order = a.order;
    sz->scalar_type = A->scalar_type;
    return SPMM_OK;
}

template <typename I, typename S>
int boo_emit_impl(const BooArgs &a, BooWs &w, spmm_boo_dev *o, cudaStream_t s) {
    const spmm_csr_dev *A = a.A;
    const int64_t rows = A->rows, cols = A->cols, nnz = A->nnz;
    const I *indptr = (const I *)A->indptr;
    const I *indices = (const I *)A->indices;
    const S *values = (const S *)A->values;
    const int T = 256;
    BuildCounters h;
    SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    const int64_t n_rg = o->n_rg, n_cg = o->n_cg;
    if ((int64_t)h.n_rg != n_rg || (int64_t)h.n_cg != n_cg || h.nb != (uint32_t)o->nb ||
        h.nnz_c != (uint32_t)o->nnz_c)
        return SPMM_EINVAL;  // workspace does not hold this build's analysis

    SPMM_CUDA_TRY(cudaMemcpyAsync(o->row_grp_ptr, w.rgp, sizeof(int32_t) * (size_t)(n_rg + 1),
                                  cudaMemcpyDeviceToDevice, s));
    SPMM_CUDA_TRY(cudaMemcpyAsync(o->col_grp_ptr, w.cgp, sizeof(int32_t) * (size_t)(n_cg + 1),
                                  cudaMemcpyDeviceToDevice, s));
    if (rows) SPMM_CUDA_TRY(cudaMemcpyAsync(o->row_ids, w.rids, sizeof(int32_t) * (size_t)rows,
                                            cudaMemcpyDeviceToDevice, s));
    if (cols) SPMM_CUDA_TRY(cudaMemcpyAsync(o->col_ids, w.cids, sizeof(int32_t) * (size_t)cols,
                                            cudaMemcpyDeviceToDevice, s));
    const uint32_t nb = (uint32_t)o->nb, nnz_c = (uint32_t)o->nnz_c;
    const int64_t n_spill = nnz - (int64_t)nnz_c;
    if (nnz == 0) {
        SPMM_CUDA_TRY(cudaMemsetAsync(o->blk_nz_ptr, 0, sizeof(int32_t), s));
        SPMM_CUDA_TRY(cudaMemsetAsync(o->rem_indptr, 0, sizeof(int32_t) * (size_t)(rows + 1), s));
        return SPMM_OK;
    }
    const uint32_t n_cand = h.n_cand;
    emit_blocks_kernel<<<grid_for(n_cand, T), T, 0, s>>>(w.k0, w.bstart, n_cand, (const uint32_t *)w.tmp_col,
                                                         w.keep, w.kcnt, n_cg, w.cgp, nb, nnz_c,
                                                         o->blk_row_grp, o->blk_col_grp,
                                                         o->blk_nz_ptr, o->blk_shift);
    SPMM_LAUNCH_CHECK();
    SPMM_CUDA_TRY(cudaMemsetAsync(w.spill, 0, sizeof(uint32_t) * (size_t)(nnz + 1), s));
    emit_entries_kernel<I, S><<<grid_for(nnz, T), T, 0, s>>>(
        w.v0, nnz, w.flag, w.bstart, (const uint32_t *)w.tmp_col, w.kcnt, indices, values, w.row_of,
        w.rpos, w.cpos, a.cl, w.cgp, o->nz_idx, (S *)o->nz_val, w.spill);
    SPMM_LAUNCH_CHECK();
    // spill positions in CSR order; keep the raw flags in `bstart` (free now)
    SPMM_CUDA_TRY(cudaMemcpyAsync(w.bstart, w.spill, sizeof(uint32_t) * (size_t)(nnz + 1),
                                  cudaMemcpyDeviceToDevice, s));
    SPMM_TRY(exclusive_scan<uint32_t>(w.spill, w.spill, nnz + 1, w.scan_temp, nullptr, s));
    const uint32_t *spill_flag = w.bstart;
    const uint32_t *spos = w.spill;
    if (a.policy == SPMM_BOO_TAIL_BATCH) {
        SPMM_CUDA_TRY(cudaMemsetAsync(o->rem_indptr, 0, sizeof(int32_t) * (size_t)(rows + 1), s));
        if (n_spill)
            emit_spill_kernel<int32_t, I, S><<<grid_for(nnz, T), T, 0, s>>>(
                spill_flag, spos, nnz, w.row_of, nullptr, indices, values, o->tail_row, o->tail_col,
                (S *)o->tail_val);
        SPMM_LAUNCH_CHECK();
        return SPMM_OK;
    }
    rem_indptr_kernel<I, int32_t><<<grid_for(rows + 1, T), T, 0, s>>>(indptr, rows, spos, o->rem_indptr);
    SPMM_LAUNCH_CHECK();
    if (n_spill == 0) return SPMM_OK;
    if (!h.unsorted) {
        // canonical CSR: spilled entries in CSR order are already (row, col)-sorted
        emit_spill_kernel<int32_t, I, S><<<grid_for(nnz, T), T, 0, s>>>(
            spill_flag, spos, nnz, w.row_of, nullptr, indices, values, nullptr, o->rem_col_ind,
            (S *)o->rem_vals);
        SPMM_LAUNCH_CHECK();
        return SPMM_OK;
    }
    // general input: sort the remainder by (row, col, value), value first (LSD)
    S *tval = (S *)w.tmp_val;
    emit_spill_kernel<int32_t, I, S><<<grid_for(nnz, T), T, 0, s>>>(
        spill_flag, spos, nnz, w.row_of, nullptr, indices, values, nullptr, w.tmp_col, tval);
    SPMM_LAUNCH_CHECK();
    int32_t *prow = (int32_t *)w.flag;  // row of each staged remainder entry (flag is free now)
    emit_spill_kernel<int32_t, I, int32_t><<<grid_for(nnz, T), T, 0, s>>>(
        spill_flag, spos, nnz, w.row_of, w.row_of, indices, w.row_of, nullptr, prow,
        (int32_t *)w.v1);
    SPMM_LAUNCH_CHECK();
    SPMM_TRY(sort_remainder<int32_t, S>(rows, cols, n_spill, prow, w.tmp_col, tval, w.k0, w.v0, w.k1,
                                        w.v1, w.sort_temp, o->rem_col_ind, (S *)o->rem_vals, s));
    return SPMM_OK;
}

}  // namespace
}  // namespace spmm

using namespace spmm;

extern "C" size_t spmm_boo_build_workspace_size(int64_t rows, int64_t cols, int64_t nnz) {
    if (rows < 0 || cols < 0 || nnz < 0) return 0;
    return boo_ws_layout<false>(rows, cols, nnz, nullptr, 0, nullptr) + 256;
}

extern "C" int spmm_boo_build_analyze(const spmm_csr_dev *A, const int32_t *row_labels,
                                      const int32_t *col_labels, int policy, int64_t threshold,
                                      int nz_order, void *workspace, size_t workspace_bytes,
                                      spmm_boo_dev *sizes, spmm_stream_t stream) {
    BooArgs a{A, row_labels, col_labels, policy, threshold, nz_order};
    SPMM_TRY(validate_args(a));
    if (!sizes || !workspace) return SPMM_EINVAL;
    if (workspace_bytes < spmm_boo_build_workspace_size(A->rows, A->cols, A->nnz))
        return SPMM_EWORKSPACE;
    BooWs w;
    boo_ws_layout<true>(A->rows, A->cols, A->nnz, workspace, workspace_bytes, &w);
    cudaStream_t s = (cudaStream_t)stream;
    return dispatch_is(A, [&](auto i, auto v) {
        return boo_analyze_impl<decltype(i), decltype(v)>(a, w, sizes, s);
    });
}

extern "C" int spmm_boo_build_emit(const spmm_csr_dev *A, const int32_t *row_labels,
                                   const int32_t *col_labels, int policy, int64_t threshold,
                                   int nz_order, void *workspace, size_t workspace_bytes,
                                   spmm_boo_dev *out, spmm_stream_t stream) {
    BooArgs a{A, row_labels, col_labels, policy, threshold, nz_order};
    SPMM_TRY(validate_args(a));
    if (!out || !workspace) return SPMM_EINVAL;
    if (workspace_bytes < spmm_boo_build_workspace_size(A->rows, A->cols, A->nnz))
        return SPMM_EWORKSPACE;
    if (!out->row_grp_ptr || !out->col_grp_ptr || !out->blk_nz_ptr || !out->rem_indptr)
        return SPMM_EINVAL;
    BooWs w;
    boo_ws_layout<true>(A->rows, A->cols, A->nnz, workspace, workspace_bytes, &w);
    cudaStream_t s = (cudaStream_t)stream;
    return dispatch_is(A, [&](auto i, auto v) {
        return boo_emit_impl<decltype(i), decltype(v)>(a, w, out, s);
    });
}
