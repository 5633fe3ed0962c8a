// build_common.cuh -- kernels shared by the BOO and PBR GPU builders.
#pragma once

#include "common.cuh"

namespace spmm {
namespace {

// Device-side counters of one build; read back by the analyze phase.
struct BuildCounters {
    unsigned long long n_rg, n_cg;       // BOO: max label + 1
    unsigned long long max_nr, max_nc, max_nnz_blk;
    unsigned int err_label, err_u16, err_index, unsorted, err_dup, pad0;
    uint32_t n_cand, nb, nnz_c, n_spill;
};

__device__ __forceinline__ uint32_t ceil_log2_dev(uint32_t v) {
    // smallest s with (1 << s) >= v; 0 or 1 -> 0 (boo_matrix.cpp:12-16)
    return v <= 1 ? 0u : 32u - (uint32_t)__clz(v - 1);
}

template <typename I>
__global__ void check_indptr_kernel(const I *__restrict__ indptr, int64_t rows, int64_t nnz,
                                    BuildCounters *cnt) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r <= rows;
         r += (int64_t)gridDim.x * blockDim.x) {
        int64_t v = (int64_t)indptr[r];
        bool bad = (r == 0 && v != 0) || (r == rows && v != nnz) ||
                   (r < rows && (int64_t)indptr[r + 1] < v) || v < 0 || v > nnz;
        if (bad) atomicOr(&cnt->err_index, 1u);
    }
}

// One warp per CSR row: records the row of every nonzero, checks column
// bounds, and flags rows whose columns are not strictly increasing (unsorted
// or duplicate entries).
template <typename I>
__global__ void row_of_kernel(const I *__restrict__ indptr, const I *__restrict__ indices,
                              int64_t rows, int64_t cols, int32_t *__restrict__ row_of,
                              BuildCounters *cnt) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    bool unsorted = false, bad = false;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const int64_t b = indptr[r], e = indptr[r + 1];
        for (int64_t j = b + lane; j < e; j += 32) {
            row_of[j] = (int32_t)r;
            const int64_t c = (int64_t)indices[j];
            if (c < 0 || c >= cols) bad = true;
            if (j > b && (int64_t)indices[j - 1] >= c) unsorted = true;
        }
    }
    if (__any_sync(kFullMask, bad) && lane == 0) atomicOr(&cnt->err_index, 1u);
    if (__any_sync(kFullMask, unsorted) && lane == 0) atomicOr(&cnt->unsorted, 1u);
}

// flag[i] = 1 where sorted key i starts a new block (key >> shift differs).
__global__ void seg_flag_kernel(const uint64_t *__restrict__ keys, int64_t n, int shift,
                                uint32_t *__restrict__ flag) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= n;
         i += (int64_t)gridDim.x * blockDim.x)
        flag[i] = (i < n) && (i == 0 || (keys[i] >> shift) != (keys[i - 1] >> shift));
}

// In place: exclusive-scanned head flags -> block id of every entry;
// bstart[block] = first entry.
__global__ void seg_start_kernel(const uint64_t *__restrict__ keys, int64_t n, int shift,
                                 uint32_t *__restrict__ scanned, uint32_t *__restrict__ bstart) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        bool head = (i == 0 || (keys[i] >> shift) != (keys[i - 1] >> shift));
        uint32_t s = scanned[i];
        if (head) bstart[s] = (uint32_t)i;
        scanned[i] = head ? s : s - 1;
    }
}

// Compacts flagged CSR positions (spos = exclusive scan of the flags).
template <typename IO, typename I, typename S>
__global__ void emit_spill_kernel(const uint32_t *__restrict__ spill_flag,
                                  const uint32_t *__restrict__ spos, int64_t nnz,
                                  const int32_t *__restrict__ row_src,
                                  const int32_t *__restrict__ col_src,  // null: use indices
                                  const I *__restrict__ indices, const S *__restrict__ values,
                                  IO *__restrict__ out_row, IO *__restrict__ out_col,
                                  S *__restrict__ out_val) {
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < nnz;
         j += (int64_t)gridDim.x * blockDim.x) {
        if (!spill_flag[j]) continue;
        const uint32_t p = spos[j];
        if (out_row) out_row[p] = (IO)row_src[j];
        out_col[p] = col_src ? (IO)col_src[j] : (IO)indices[j];
        out_val[p] = values[j];
    }
}

// rem_indptr[r] = spos[indptr[r]]: valid when every spilled entry stays in
// its own CSR row.
template <typename I, typename IO>
__global__ void rem_indptr_kernel(const I *__restrict__ indptr, int64_t rows,
                                  const uint32_t *__restrict__ spos, IO *__restrict__ rem_indptr) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r <= rows;
         r += (int64_t)gridDim.x * blockDim.x)
        rem_indptr[r] = (IO)spos[(int64_t)indptr[r]];
}

template <typename S>
__global__ void value_keys_kernel(const S *__restrict__ vals, int64_t n,
                                  uint64_t *__restrict__ keys, uint32_t *__restrict__ perm) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n;
         p += (int64_t)gridDim.x * blockDim.x) {
        keys[p] = order_key(vals[p]);
        perm[p] = (uint32_t)p;
    }
}

__global__ void rowcol_keys_kernel(const uint32_t *__restrict__ perm,
                                   const int32_t *__restrict__ rows_of,
                                   const int32_t *__restrict__ cols_of, int col_bits, int64_t n,
                                   uint64_t *__restrict__ keys) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n;
         q += (int64_t)gridDim.x * blockDim.x) {
        uint32_t p = perm[q];
        keys[q] = ((uint64_t)(uint32_t)rows_of[p] << col_bits) | (uint64_t)(uint32_t)cols_of[p];
    }
}

template <typename IO, typename S>
__global__ void gather_colval_kernel(const uint32_t *__restrict__ perm, int64_t n,
                                     const int32_t *__restrict__ col_in, const S *__restrict__ val_in,
                                     IO *__restrict__ col_out, S *__restrict__ val_out) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n;
         q += (int64_t)gridDim.x * blockDim.x) {
        uint32_t p = perm[q];
        col_out[q] = (IO)col_in[p];
        val_out[q] = val_in[p];
    }
}

__global__ void count_rows_kernel(const int32_t *__restrict__ row_of_p, int64_t n,
                                  uint32_t *__restrict__ counts) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n;
         p += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(&counts[row_of_p[p]], 1u);
}

template <typename IO>
__global__ void copy_u32_kernel(const uint32_t *__restrict__ in, int64_t n, IO *__restrict__ out) {
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < n;
         p += (int64_t)gridDim.x * blockDim.x)
        out[p] = (IO)in[p];
}

// Sorts n staged remainder entries (prow, pcol, pval) by (row, col, value)
// -- the order std::sort gives per-row (col, value) pairs -- and writes the
// column / value arrays.  Two stable LSD sorts: value first, then (row, col).
template <typename IO, typename S>
int sort_remainder(int64_t rows, int64_t cols, int64_t n, const int32_t *prow, const int32_t *pcol,
                   const S *pval, uint64_t *k0, uint32_t *v0, uint64_t *k1, uint32_t *v1,
                   uint32_t *sort_temp, IO *out_col, S *out_val, cudaStream_t s) {
    if (n == 0) return SPMM_OK;
    const int T = 256;
    value_keys_kernel<S><<<grid_for(n, T), T, 0, s>>>(pval, n, k0, v0);
    SPMM_LAUNCH_CHECK();
    bool first;
    SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(k0, v0, k1, v1, n, 8 * (int)sizeof(S), sort_temp,
                                                  &first, s));
    uint32_t *perm = first ? v0 : v1;
    uint64_t *kk = first ? k0 : k1;
    uint64_t *kk2 = first ? k1 : k0;
    uint32_t *pp2 = first ? v1 : v0;
    const int col_bits = bit_width_u64((uint64_t)(cols > 0 ? cols - 1 : 0));
    const int key_bits = bit_width_u64((uint64_t)(rows > 0 ? rows - 1 : 0)) + col_bits;
    rowcol_keys_kernel<<<grid_for(n, T), T, 0, s>>>(perm, prow, pcol, col_bits, n, kk);
    SPMM_LAUNCH_CHECK();
    SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(kk, perm, kk2, pp2, n, key_bits, sort_temp, &first, s));
    gather_colval_kernel<IO, S><<<grid_for(n, T), T, 0, s>>>(first ? perm : pp2, n, pcol, pval,
                                                             out_col, out_val);
    SPMM_LAUNCH_CHECK();
    return SPMM_OK;
}

template <typename F>
int dispatch_is(const spmm_csr_dev *A, F &&f) {
    if (A->index_type == SPMM_INDEX_I32) {
        if (A->scalar_type == SPMM_F32) return f((int32_t)0, 0.0f);
        return f((int32_t)0, 0.0);
    }
    if (A->scalar_type == SPMM_F32) return f((int64_t)0, 0.0f);
    return f((int64_t)0, 0.0);
}

inline int validate_csr(const spmm_csr_dev *A) {
    if (!A) return SPMM_EINVAL;
    if (A->rows < 0 || A->cols < 0 || A->nnz < 0) return SPMM_EINVAL;
    if (A->rows > 0x7fffffffLL || A->cols > 0x7fffffffLL || A->nnz > 0x7ffffffeLL)
        return SPMM_EUNSUPPORTED;
    if (A->index_type != SPMM_INDEX_I32 && A->index_type != SPMM_INDEX_I64) return SPMM_EINVAL;
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return SPMM_EINVAL;
    if (!A->indptr || (A->nnz && (!A->indices || !A->values))) return SPMM_EINVAL;
    return SPMM_OK;
}

}  // namespace
}  // namespace spmm
