// build_pbr.cu -- GPU construction of the PBR format from a device CSR.
//
// Reproduces the reference builder csr_to_pbr (torch_fast_spdmm/pbr_matrix/
// pbr_matrix.cpp:333-448):
//   * block (stripe = row / BR, block column = col / BC), bit
//     (row % BR) * BC + col % BC of a 64-bit code (:372-388)
//   * block values in CSR traversal order (:389) -> stable radix sort of the
//     nonzeros by block key
//   * keep iff popcount(code) >= min_nnz_per_block (:397-406); offsets advance
//     by popcount
//   * a spilled block's k-th set bit (bit order) takes its k-th value
//     (traversal order) into the remainder (:407-416); remainder rows sorted by
//     (col, value) (:425-439).
// Blocks are emitted in (stripe, block column) order; the reference's order
// inside a stripe is std::unordered_map iteration order (:396), which no other
// implementation can reproduce.  Input with duplicate (row, col) entries is
// rejected (SPMM_EDUPLICATE): the reference appends every duplicate value to
// block_data while advancing block_offsets by popcount, which leaves the
// format inconsistent with itself.
#include "build_common.cuh"

namespace spmm {
namespace {

struct PbrWs {
    BuildCounters *cnt;
    int32_t *row_of;                     // nnz
    uint64_t *k0, *k1;                   // nnz
    uint32_t *v0, *v1;                   // nnz
    uint32_t *sort_temp;
    uint32_t *flag;                      // nnz+1 : head flags -> block of entry
    uint32_t *bstart;                    // nnz+1
    uint64_t *code;                      // nnz   : code of each candidate block
    uint32_t *keep;                      // nnz+1 : raw keep flags
    uint32_t *kidx;                      // nnz+1 : kept index (scan)
    uint32_t *kcnt;                      // nnz+1 : kept popcounts -> data offset (scan)
    uint32_t *spill;                     // nnz+1 : spill flag per CSR position
    uint32_t *spos;                      // nnz+1 : its exclusive scan
    int32_t *arow, *acol;                // nnz   : row / col a spilled entry is assigned to
    uint32_t *rcount;                    // rows+1: remainder row counts (general path)
    uint32_t *scan_temp;
    int32_t *tmp_row, *tmp_col;          // nnz
    double *tmp_val;                     // nnz
};

template <bool CARVE>
size_t pbr_ws_layout(int64_t rows, int64_t nnz, void *base, size_t cap, PbrWs *ws) {
    int64_t big = nnz + 1 > rows + 1 ? nnz + 1 : rows + 1;
    Arena a(base, cap);
    size_t used = 0;
#define CARVE_(field, T, n)                       \
    do {                                          \
        if (CARVE) ws->field = a.take<T>(n);      \
        else arena_count<T>(used, n);             \
    } while (0)
    CARVE_(cnt, BuildCounters, 1);
    CARVE_(row_of, int32_t, nnz);
    CARVE_(k0, uint64_t, nnz);
    CARVE_(k1, uint64_t, nnz);
    CARVE_(v0, uint32_t, nnz);
    CARVE_(v1, uint32_t, nnz);
    CARVE_(sort_temp, uint32_t, radix_temp_elems(nnz));
    CARVE_(flag, uint32_t, nnz + 1);
    CARVE_(bstart, uint32_t, nnz + 1);
    CARVE_(code, uint64_t, nnz);
    CARVE_(keep, uint32_t, nnz + 1);
    CARVE_(kidx, uint32_t, nnz + 1);
    CARVE_(kcnt, uint32_t, nnz + 1);
    CARVE_(spill, uint32_t, nnz + 1);
    CARVE_(spos, uint32_t, nnz + 1);
    CARVE_(arow, int32_t, nnz);
    CARVE_(acol, int32_t, nnz);
    CARVE_(rcount, uint32_t, rows + 1);
    CARVE_(scan_temp, uint32_t, scan_temp_elems(big) + 2);
    CARVE_(tmp_row, int32_t, nnz);
    CARVE_(tmp_col, int32_t, nnz);
    CARVE_(tmp_val, double, nnz);
#undef CARVE_
    return CARVE ? a.used : used;
}

template <typename I>
__global__ void pbr_keys_kernel(const I *__restrict__ indices, const int32_t *__restrict__ row_of,
                                int64_t nnz, int64_t br, int64_t bc, int64_t n_bcol,
                                uint64_t *__restrict__ keys, uint32_t *__restrict__ vals) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < nnz;
         j += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = row_of[j], c = (int64_t)indices[j];
        keys[j] = (uint64_t)((r / br) * n_bcol + c / bc);
        vals[j] = (uint32_t)j;
    }
}

// One thread per candidate block: OR of the entries' bits, duplicate check,
// keep decision.
template <typename I>
__global__ void pbr_codes_kernel(const uint32_t *__restrict__ vals, const uint32_t *__restrict__ bstart,
                                 uint32_t n_cand, int64_t nnz, const int32_t *__restrict__ row_of,
                                 const I *__restrict__ indices, int64_t br, int64_t bc,
                                 int min_nnz, uint64_t *__restrict__ code, uint32_t *__restrict__ keep,
                                 uint32_t *__restrict__ kcnt, BuildCounters *cnt) {
    bool dup = false;
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b <= (int64_t)n_cand;
         b += (int64_t)gridDim.x * blockDim.x) {
        if (b == (int64_t)n_cand) { keep[b] = 0; kcnt[b] = 0; continue; }
        const uint32_t s = bstart[b];
        const uint32_t e = (b + 1 < (int64_t)n_cand) ? bstart[b + 1] : (uint32_t)nnz;
        uint64_t c = 0;
        for (uint32_t i = s; i < e; ++i) {
            const uint32_t j = vals[i];
            const int64_t bit = ((int64_t)row_of[j] % br) * bc + (int64_t)indices[j] % bc;
            c |= 1ull << bit;
        }
        const uint32_t pc = (uint32_t)__popcll(c);
        if (pc != e - s) dup = true;
        code[b] = c;
        const bool k = (int)pc >= min_nnz;
        keep[b] = k;
        kcnt[b] = k ? pc : 0;
    }
    if (dup) atomicOr(&cnt->err_dup, 1u);
}

template <typename IO>
__global__ void pbr_emit_blocks_kernel(const uint64_t *__restrict__ keys,
                                       const uint32_t *__restrict__ bstart, uint32_t n_cand,
                                       const uint64_t *__restrict__ code,
                                       const uint32_t *__restrict__ keep,
                                       const uint32_t *__restrict__ kidx,
                                       const uint32_t *__restrict__ kofs, int64_t br, int64_t bc,
                                       int64_t n_bcol, uint32_t nb, uint32_t nnz_c,
                                       uint64_t *__restrict__ codes, IO *__restrict__ coords,
                                       IO *__restrict__ offsets) {
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < (int64_t)n_cand;
         b += (int64_t)gridDim.x * blockDim.x) {
        if (!keep[b]) continue;
        const uint32_t kb = kidx[b];
        const int64_t key = (int64_t)keys[bstart[b]];
        codes[kb] = code[b];
        coords[2 * (int64_t)kb] = (IO)((key / n_bcol) * br);
        coords[2 * (int64_t)kb + 1] = (IO)((key % n_bcol) * bc);
        offsets[kb] = (IO)kofs[b];
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) offsets[nb] = (IO)nnz_c;
}

// The k-th set bit of v (k < popcount(v)).
__device__ __forceinline__ int kth_set_bit(uint64_t v, uint32_t k) {
    for (uint32_t t = 0; t < k; ++t) v &= v - 1;
    return __ffsll((long long)v) - 1;
}

template <typename S>
__global__ void pbr_emit_entries_kernel(const uint64_t *__restrict__ keys,
                                        const uint32_t *__restrict__ vals, int64_t nnz,
                                        const uint32_t *__restrict__ blk_of,
                                        const uint32_t *__restrict__ bstart,
                                        const uint64_t *__restrict__ code,
                                        const uint32_t *__restrict__ keep,
                                        const uint32_t *__restrict__ kofs,
                                        const S *__restrict__ values, int64_t br, int64_t bc,
                                        int64_t n_bcol, S *__restrict__ data,
                                        uint32_t *__restrict__ spill, int32_t *__restrict__ arow,
                                        int32_t *__restrict__ acol) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nnz;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t b = blk_of[i];
        const uint32_t j = vals[i];
        const uint32_t k = (uint32_t)(i - bstart[b]);
        if (keep[b]) {
            data[kofs[b] + k] = values[j];
        } else {
            const int bit = kth_set_bit(code[b], k);
            const int64_t key = (int64_t)keys[i];
            arow[j] = (int32_t)((key / n_bcol) * br + bit / bc);
            acol[j] = (int32_t)((key % n_bcol) * bc + bit % bc);
            spill[j] = 1u;
        }
    }
}

struct PbrArgs {
    const spmm_csr_dev *A;
    int64_t br, bc;
    int min_nnz;
};

int pbr_validate(const PbrArgs &a) {
    SPMM_TRY(validate_csr(a.A));
    if (a.br <= 0 || a.bc <= 0 || a.br * a.bc > 64) return SPMM_EINVAL;
    return SPMM_OK;
}

template <typename I, typename S>
int pbr_analyze_impl(const PbrArgs &a, PbrWs &w, spmm_pbr_dev *sz, cudaStream_t s) {
    const spmm_csr_dev *A = a.A;
    const int64_t rows = A->rows, cols = A->cols, nnz = A->nnz;
    const I *indptr = (const I *)A->indptr;
    const I *indices = (const I *)A->indices;
    const int T = 256;
    SPMM_CUDA_TRY(cudaMemsetAsync(w.cnt, 0, sizeof(BuildCounters), s));
    check_indptr_kernel<I><<<grid_for(rows + 1, T), T, 0, s>>>(indptr, rows, nnz, w.cnt);
    SPMM_LAUNCH_CHECK();
    BuildCounters h;
    SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    if (h.err_index) return SPMM_EINVAL;
    uint32_t nb = 0, nnz_c = 0;
    if (nnz > 0) {
        row_of_kernel<I><<<grid_for(rows * 32, T), T, 0, s>>>(indptr, indices, rows, cols, w.row_of, w.cnt);
        SPMM_LAUNCH_CHECK();
        SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
        SPMM_CUDA_TRY(cudaStreamSynchronize(s));
        if (h.err_index) return SPMM_EINVAL;
        const int64_t n_bcol = (cols + a.bc - 1) / a.bc;
        const int64_t n_strp = (rows + a.br - 1) / a.br;
        const int key_bits = bit_width_u64((uint64_t)(n_strp * n_bcol - 1));
        pbr_keys_kernel<I><<<grid_for(nnz, T), T, 0, s>>>(indices, w.row_of, nnz, a.br, a.bc, n_bcol,
                                                          w.k0, w.v0);
        SPMM_LAUNCH_CHECK();
        bool first;
        SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(w.k0, w.v0, w.k1, w.v1, nnz, key_bits,
                                                      w.sort_temp, &first, s));
        if (!first) {
            SPMM_CUDA_TRY(cudaMemcpyAsync(w.k0, w.k1, sizeof(uint64_t) * (size_t)nnz,
                                          cudaMemcpyDeviceToDevice, s));
            SPMM_CUDA_TRY(cudaMemcpyAsync(w.v0, w.v1, sizeof(uint32_t) * (size_t)nnz,
                                          cudaMemcpyDeviceToDevice, s));
        }
        seg_flag_kernel<<<grid_for(nnz + 1, T), T, 0, s>>>(w.k0, nnz, 0, w.flag);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(exclusive_scan<uint32_t>(w.flag, w.flag, nnz + 1, w.scan_temp, &w.cnt->n_cand, s));
        seg_start_kernel<<<grid_for(nnz, T), T, 0, s>>>(w.k0, nnz, 0, w.flag, w.bstart);
        SPMM_LAUNCH_CHECK();
        SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
        SPMM_CUDA_TRY(cudaStreamSynchronize(s));
        const uint32_t n_cand = h.n_cand;
        pbr_codes_kernel<I><<<grid_for((int64_t)n_cand + 1, T), T, 0, s>>>(
            w.v0, w.bstart, n_cand, nnz, w.row_of, indices, a.br, a.bc, a.min_nnz, w.code, w.keep,
            w.kcnt, w.cnt);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(exclusive_scan<uint32_t>(w.keep, w.kidx, (int64_t)n_cand + 1, w.scan_temp, &w.cnt->nb, s));
        SPMM_TRY(exclusive_scan<uint32_t>(w.kcnt, w.kcnt, (int64_t)n_cand + 1, w.scan_temp,
                                          &w.cnt->nnz_c, s));
        SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
        SPMM_CUDA_TRY(cudaStreamSynchronize(s));
        if (h.err_dup) return SPMM_EDUPLICATE;
        nb = h.nb;
        nnz_c = h.nnz_c;
    }
    sz->rows = rows;
    sz->cols = cols;
    sz->block_rows = a.br;
    sz->block_cols = a.bc;
    sz->total_nnz = nnz;
    sz->nb = nb;
    sz->nnz_c = nnz_c;
    sz->rem_nnz = nnz - (int64_t)nnz_c;
    sz->scalar_type = A->scalar_type;
    return SPMM_OK;
}

template <typename I, typename S, typename IO>
int pbr_emit_impl(const PbrArgs &a, PbrWs &w, spmm_pbr_dev *o, cudaStream_t s) {
    const spmm_csr_dev *A = a.A;
    const int64_t rows = A->rows, cols = A->cols, nnz = A->nnz;
    const I *indptr = (const I *)A->indptr;
    const I *indices = (const I *)A->indices;
    const S *values = (const S *)A->values;
    const int T = 256;
    BuildCounters h;
    SPMM_CUDA_TRY(cudaMemcpyAsync(&h, w.cnt, sizeof(h), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    const uint32_t nb = (uint32_t)o->nb, nnz_c = (uint32_t)o->nnz_c;
    if (nnz > 0 && (h.nb != nb || h.nnz_c != nnz_c)) return SPMM_EINVAL;
    IO *offsets = (IO *)o->offsets;
    IO *rem_indptr = (IO *)o->rem_indptr;
    if (nnz == 0) {
        SPMM_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(IO), s));
        SPMM_CUDA_TRY(cudaMemsetAsync(rem_indptr, 0, sizeof(IO) * (size_t)(rows + 1), s));
        return SPMM_OK;
    }
    const int64_t n_bcol = (cols + a.bc - 1) / a.bc;
    const uint32_t n_cand = h.n_cand;
    pbr_emit_blocks_kernel<IO><<<grid_for(n_cand, T), T, 0, s>>>(
        w.k0, w.bstart, n_cand, w.code, w.keep, w.kidx, w.kcnt, a.br, a.bc, n_bcol, nb, nnz_c,
        o->codes, (IO *)o->coords, offsets);
    SPMM_LAUNCH_CHECK();
    SPMM_CUDA_TRY(cudaMemsetAsync(w.spill, 0, sizeof(uint32_t) * (size_t)(nnz + 1), s));
    pbr_emit_entries_kernel<S><<<grid_for(nnz, T), T, 0, s>>>(
        w.k0, w.v0, nnz, w.flag, w.bstart, w.code, w.keep, w.kcnt, values, a.br, a.bc, n_bcol,
        (S *)o->data, w.spill, w.arow, w.acol);
    SPMM_LAUNCH_CHECK();
    const int64_t n_spill = nnz - (int64_t)nnz_c;
    SPMM_TRY(exclusive_scan<uint32_t>(w.spill, w.spos, nnz + 1, w.scan_temp, nullptr, s));
    if (!h.unsorted) {
        // canonical CSR: a spilled entry's assigned (row, col) is its own, and
        // CSR order is (row, col) order
        rem_indptr_kernel<I, IO><<<grid_for(rows + 1, T), T, 0, s>>>(indptr, rows, w.spos, rem_indptr);
        SPMM_LAUNCH_CHECK();
        if (n_spill)
            emit_spill_kernel<IO, I, S><<<grid_for(nnz, T), T, 0, s>>>(
                w.spill, w.spos, nnz, w.row_of, nullptr, indices, values, nullptr,
                (IO *)o->rem_col_ind, (S *)o->rem_vals);
        SPMM_LAUNCH_CHECK();
        return SPMM_OK;
    }
    // general input: stage (assigned row, assigned col, value), count rows, sort
    S *tval = (S *)w.tmp_val;
    SPMM_CUDA_TRY(cudaMemsetAsync(w.rcount, 0, sizeof(uint32_t) * (size_t)(rows + 1), s));
    if (n_spill) {
        emit_spill_kernel<int32_t, I, S><<<grid_for(nnz, T), T, 0, s>>>(
            w.spill, w.spos, nnz, w.arow, w.acol, indices, values, w.tmp_row, w.tmp_col, tval);
        SPMM_LAUNCH_CHECK();
        count_rows_kernel<<<grid_for(n_spill, T), T, 0, s>>>(w.tmp_row, n_spill, w.rcount);
        SPMM_LAUNCH_CHECK();
    }
    SPMM_TRY(exclusive_scan<uint32_t>(w.rcount, w.rcount, rows + 1, w.scan_temp, nullptr, s));
    copy_u32_kernel<IO><<<grid_for(rows + 1, T), T, 0, s>>>(w.rcount, rows + 1, rem_indptr);
    SPMM_LAUNCH_CHECK();
    return sort_remainder<IO, S>(rows, cols, n_spill, w.tmp_row, w.tmp_col, tval, w.k0, w.v0, w.k1,
                                 w.v1, w.sort_temp, (IO *)o->rem_col_ind, (S *)o->rem_vals, s);
}

}  // namespace
}  // namespace spmm

using namespace spmm;

extern "C" size_t spmm_pbr_build_workspace_size(int64_t rows, int64_t cols, int64_t nnz) {
    (void)cols;
    if (rows < 0 || cols < 0 || nnz < 0) return 0;
    return pbr_ws_layout<false>(rows, nnz, nullptr, 0, nullptr) + 256;
}

extern "C" int spmm_pbr_build_analyze(const spmm_csr_dev *A, int64_t block_rows, int64_t block_cols,
                                      int min_nnz_per_block, void *workspace, size_t workspace_bytes,
                                      spmm_pbr_dev *sizes, spmm_stream_t stream) {
    PbrArgs a{A, block_rows, block_cols, min_nnz_per_block};
    SPMM_TRY(pbr_validate(a));
    if (!sizes || !workspace) return SPMM_EINVAL;
    if (workspace_bytes < spmm_pbr_build_workspace_size(A->rows, A->cols, A->nnz)) return SPMM_EWORKSPACE;
    PbrWs w;
    pbr_ws_layout<true>(A->rows, A->nnz, workspace, workspace_bytes, &w);
    cudaStream_t s = (cudaStream_t)stream;
    return dispatch_is(A, [&](auto i, auto v) {
        return pbr_analyze_impl<decltype(i), decltype(v)>(a, w, sizes, s);
    });
}

extern "C" int spmm_pbr_build_emit(const spmm_csr_dev *A, int64_t block_rows, int64_t block_cols,
                                   int min_nnz_per_block, void *workspace, size_t workspace_bytes,
                                   spmm_pbr_dev *out, spmm_stream_t stream) {
    PbrArgs a{A, block_rows, block_cols, min_nnz_per_block};
    SPMM_TRY(pbr_validate(a));
    if (!out || !workspace) return SPMM_EINVAL;
    if (workspace_bytes < spmm_pbr_build_workspace_size(A->rows, A->cols, A->nnz)) return SPMM_EWORKSPACE;
    if (!out->offsets || !out->rem_indptr) return SPMM_EINVAL;
    if (out->index_type != SPMM_INDEX_I32 && out->index_type != SPMM_INDEX_I64) return SPMM_EINVAL;
    PbrWs w;
    pbr_ws_layout<true>(A->rows, A->nnz, workspace, workspace_bytes, &w);
    cudaStream_t s = (cudaStream_t)stream;
    return dispatch_is(A, [&](auto i, auto v) {
        using I = decltype(i);
        using S = decltype(v);
        if (out->index_type == SPMM_INDEX_I32) return pbr_emit_impl<I, S, int32_t>(a, w, out, s);
        return pbr_emit_impl<I, S, int64_t>(a, w, out, s);
    });
}
