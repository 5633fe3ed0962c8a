// convert.cu -- BOO / PBR back to CSR on the GPU (the reference's boo_to_csr,
// boo_matrix/boo_matrix.cpp:277-333, and pbr_to_csr, pbr_matrix/
// pbr_matrix.cpp:279-331).
//
// Both conversions collect every stored entry as (row, column, value) --
// blocks, then the CSR remainder, then (BOO) the COO tail -- and order each
// row by (column, value), as the reference's per-row std::sort of
// (column, value) pairs does.  Two stable radix sorts give that order: first
// by the value's order-preserving image, then by (row, column) packed in
// one word (row << column bits | column); the
// row counts scanned give indptr.  Outputs are caller-allocated, in the
// index type the caller asks for.
#include <type_traits>

#include "common.cuh"

namespace spmm {
namespace {

constexpr int kConvThreads = 256;

template <typename S>
struct ValKey;
template <>
struct ValKey<float> { using T = uint32_t; static constexpr int kBits = 32; };
template <>
struct ValKey<double> { using T = uint64_t; static constexpr int kBits = 64; };

// first i in [0, n) with a[i] > key, minus one: the segment holding `key`
template <typename I>
__device__ __forceinline__ int64_t segment_of(const I *a, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((int64_t)a[mid] <= key) lo = mid + 1; else hi = mid;
    }
    return lo - 1;
}

// BOO entry e (blocks, remainder, tail in that order) -> (row, col, value).
template <typename S>
__global__ void boo_expand_kernel(const spmm_boo_dev A, uint64_t *__restrict__ rc, S *__restrict__ val,
                                  typename ValKey<S>::T *__restrict__ vkey, uint32_t *__restrict__ id, int64_t n,
                                  int cbits) {
    const S *nz_val = (const S *)A.nz_val, *rem_val = (const S *)A.rem_vals, *tail_val = (const S *)A.tail_val;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t row, col;
        S v;
        if (e < A.nnz_c) {
            const int64_t b = segment_of(A.blk_nz_ptr, A.nb + 1, e);
            const uint32_t sh = A.blk_shift[b], idx = A.nz_idx[e];
            row = A.row_ids[A.row_grp_ptr[A.blk_row_grp[b]] + (int64_t)(idx >> sh)];
            col = A.col_ids[A.col_grp_ptr[A.blk_col_grp[b]] + (int64_t)(idx & ((1u << sh) - 1u))];
            v = nz_val[e];
        } else if (e < A.nnz_c + A.rem_nnz) {
            const int64_t k = e - A.nnz_c;
            row = segment_of(A.rem_indptr, A.rows + 1, k);
            col = A.rem_col_ind[k];
            v = rem_val[k];
        } else {
            const int64_t k = e - A.nnz_c - A.rem_nnz;
            row = A.tail_row[k];
            col = A.tail_col[k];
            v = tail_val[k];
        }
        rc[e] = ((uint64_t)row << cbits) | (uint64_t)col;
        val[e] = v;
        vkey[e] = (typename ValKey<S>::T)order_key(v);
        id[e] = (uint32_t)e;
    }
}

// PBR entry e (block values in bit order, then the remainder) -> (row, col,
// value); flags a block bit past the last row.
template <typename S, typename I>
__global__ void pbr_expand_kernel(const spmm_pbr_dev A, uint64_t *__restrict__ rc, S *__restrict__ val,
                                  typename ValKey<S>::T *__restrict__ vkey, uint32_t *__restrict__ id, int64_t n,
                                  int cbits, int *__restrict__ bad_row) {
    const I *coords = (const I *)A.coords, *offsets = (const I *)A.offsets;
    const I *rem_indptr = (const I *)A.rem_indptr, *rem_col = (const I *)A.rem_col_ind;
    const S *data = (const S *)A.data, *rem_val = (const S *)A.rem_vals;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        int64_t row, col;
        S v;
        if (e < A.nnz_c) {
            const int64_t b = segment_of(offsets, A.nb + 1, e);
            // the (e - offsets[b])-th set bit of the block's code
            uint64_t code = A.codes[b];
            for (int64_t k = e - (int64_t)offsets[b]; k > 0; --k) code &= code - 1;
            const int bit = __ffsll((long long)code) - 1;
            row = (int64_t)coords[2 * b] + bit / A.block_cols;
            col = (int64_t)coords[2 * b + 1] + bit % A.block_cols;
            if (row >= A.rows) {
                atomicExch(bad_row, 1);
                row = A.rows - 1;
            }
            v = data[e];
        } else {
            const int64_t k = e - A.nnz_c;
            row = segment_of(rem_indptr, A.rows + 1, k);
            col = rem_col[k];
            v = rem_val[k];
        }
        rc[e] = ((uint64_t)row << cbits) | (uint64_t)col;
        val[e] = v;
        vkey[e] = (typename ValKey<S>::T)order_key(v);
        id[e] = (uint32_t)e;
    }
}

template <typename K>
__global__ void gather_keys_kernel(const K *__restrict__ src, const uint32_t *__restrict__ id, K *__restrict__ dst,
                                   int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = src[id[i]];
}

template <typename S, typename I>
__global__ void emit_csr_kernel(const uint64_t *__restrict__ rc, const uint32_t *__restrict__ id,
                                const S *__restrict__ val, I *__restrict__ indices, S *__restrict__ values,
                                unsigned long long *__restrict__ counts, int64_t n, int cbits) {
    const uint64_t cmask = (1ull << cbits) - 1ull;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t k = rc[i];
        indices[i] = (I)(k & cmask);
        values[i] = val[id[i]];
        atomicAdd(counts + (k >> cbits), 1ull);
    }
}

// bits of the packed column field (at least 1)
inline int col_bits(int64_t cols) {
    const int b = bit_width_u64((uint64_t)(cols > 1 ? cols - 1 : 1));
    return b > 0 ? b : 1;
}

template <typename I>
__global__ void store_indptr_kernel(const unsigned long long *__restrict__ scanned, I *__restrict__ indptr,
                                    int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        indptr[i] = (I)scanned[i];
}

struct ConvWs {
    uint64_t *rc0, *rc1;
    void *vk0, *vk1;
    uint32_t *id0, *id1;
    void *val;
    unsigned long long *counts, *scan_tmp;
    uint32_t *sort_tmp;
    int *flag;
};

// One carve sequence for sizing (base == nullptr) and for use.
inline size_t conv_layout(int64_t rows, int64_t n, size_t sbytes, void *base, size_t cap, ConvWs *w) {
    Arena a(base, cap);
    size_t used = 0;
    auto carve = [&](auto *&dst, int64_t cnt) {
        using T = std::remove_reference_t<decltype(*dst)>;
        if (base) dst = a.take<T>(cnt);
        else arena_count<T>(used, cnt);
    };
    ConvWs t{};
    ConvWs &x = w ? *w : t;
    carve(x.rc0, n);
    carve(x.rc1, n);
    uint64_t *vk0 = nullptr, *vk1 = nullptr, *val = nullptr;   // widest value type
    carve(vk0, n);
    carve(vk1, n);
    carve(x.id0, n);
    carve(x.id1, n);
    carve(val, (int64_t)((n * (int64_t)sbytes + 7) / 8));
    carve(x.counts, rows + 1);
    carve(x.scan_tmp, scan_temp_elems(rows + 1));
    carve(x.sort_tmp, radix_temp_elems(n));
    carve(x.flag, 1);
    x.vk0 = vk0;
    x.vk1 = vk1;
    x.val = val;
    return base ? a.used : used;
}

// Sorts the expanded entries by (row, column, value) and writes the CSR.
template <typename S, typename I>
int finish_csr(const ConvWs &w, int64_t rows, int64_t cols, int64_t n, I *indptr, I *indices, S *values,
               cudaStream_t s) {
    using VK = typename ValKey<S>::T;
    const unsigned g = grid_for(n, kConvThreads);
    bool in_first = true;
    // 1. by value, carrying the entry id
    SPMM_TRY(radix_sort_pairs<VK, uint32_t>((VK *)w.vk0, w.id0, (VK *)w.vk1, w.id1, n, ValKey<S>::kBits,
                                            w.sort_tmp, &in_first, s));
    uint32_t *id = in_first ? w.id0 : w.id1;
    // 2. (row, column) keys in that order, then a stable sort by them
    gather_keys_kernel<uint64_t><<<g, kConvThreads, 0, s>>>(w.rc0, id, w.rc1, n);
    SPMM_LAUNCH_CHECK();
    uint32_t *id_other = in_first ? w.id1 : w.id0;
    const int cbits = col_bits(cols);
    const int key_bits = cbits + bit_width_u64((uint64_t)(rows > 0 ? rows - 1 : 0));
    SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(w.rc1, id, w.rc0, id_other, n, key_bits, w.sort_tmp, &in_first,
                                                  s));
    const uint64_t *rc = in_first ? w.rc1 : w.rc0;
    const uint32_t *ids = in_first ? id : id_other;
    // 3. indices, values and row counts; indptr by an exclusive scan
    SPMM_CUDA_TRY(cudaMemsetAsync(w.counts, 0, (size_t)(rows + 1) * sizeof(unsigned long long), s));
    if (n > 0) {
        emit_csr_kernel<S, I><<<g, kConvThreads, 0, s>>>(rc, ids, (const S *)w.val, indices, values, w.counts, n,
                                                         cbits);
        SPMM_LAUNCH_CHECK();
    }
    SPMM_TRY(exclusive_scan<unsigned long long>(w.counts, w.counts, rows + 1, w.scan_tmp, nullptr, s));
    store_indptr_kernel<I><<<grid_for(rows + 1, kConvThreads), kConvThreads, 0, s>>>(w.counts, indptr, rows + 1);
    SPMM_LAUNCH_CHECK();
    return SPMM_OK;
}

int64_t boo_entries(const spmm_boo_dev *A) { return A->nnz_c + A->rem_nnz + A->tail_nnz; }

template <typename S, typename I>
int boo_to_csr_impl(const spmm_boo_dev *A, const ConvWs &w, I *indptr, I *indices, S *values, cudaStream_t s) {
    const int64_t n = boo_entries(A);
    if (n > 0) {
        boo_expand_kernel<S><<<grid_for(n, kConvThreads), kConvThreads, 0, s>>>(
            *A, w.rc0, (S *)w.val, (typename ValKey<S>::T *)w.vk0, w.id0, n, col_bits(A->cols));
        SPMM_LAUNCH_CHECK();
    }
    return finish_csr<S, I>(w, A->rows, A->cols, n, indptr, indices, values, s);
}

template <typename S, typename I, typename PI>
int pbr_to_csr_impl(const spmm_pbr_dev *A, const ConvWs &w, I *indptr, I *indices, S *values, cudaStream_t s) {
    const int64_t n = A->nnz_c + A->rem_nnz;
    SPMM_CUDA_TRY(cudaMemsetAsync(w.flag, 0, sizeof(int), s));
    if (n > 0) {
        pbr_expand_kernel<S, PI><<<grid_for(n, kConvThreads), kConvThreads, 0, s>>>(
            *A, w.rc0, (S *)w.val, (typename ValKey<S>::T *)w.vk0, w.id0, n, col_bits(A->cols), w.flag);
        SPMM_LAUNCH_CHECK();
    }
    int bad = 0;
    SPMM_CUDA_TRY(cudaMemcpyAsync(&bad, w.flag, sizeof(int), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    if (bad) return SPMM_EINVAL;
    return finish_csr<S, I>(w, A->rows, A->cols, n, indptr, indices, values, s);
}

}  // namespace
}  // namespace spmm

using namespace spmm;

extern "C" size_t spmm_boo_to_csr_workspace_size(const spmm_boo_dev *A) {
    if (!A || A->rows < 0) return 0;
    const size_t sb = A->scalar_type == SPMM_F64 ? 8 : 4;
    return conv_layout(A->rows, boo_entries(A), sb, nullptr, 0, nullptr) + 256;
}

extern "C" int spmm_boo_to_csr(const spmm_boo_dev *A, void *indptr, void *indices, void *values, int index_type,
                               void *workspace, size_t workspace_bytes, spmm_stream_t stream) {
    if (!A || !indptr || A->rows < 0 || A->cols < 0) return SPMM_EINVAL;
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return SPMM_EINVAL;
    if (index_type != SPMM_INDEX_I32 && index_type != SPMM_INDEX_I64) return SPMM_EINVAL;
    const int64_t n = boo_entries(A);
    if (n > 0xFFFFFFFFLL || A->rows > 0x7fffffffLL || A->cols > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    if (n > 0 && (!indices || !values)) return SPMM_EINVAL;
    if (!workspace || workspace_bytes < spmm_boo_to_csr_workspace_size(A)) return SPMM_EWORKSPACE;
    ConvWs w;
    conv_layout(A->rows, n, A->scalar_type == SPMM_F64 ? 8 : 4, workspace, workspace_bytes, &w);
    cudaStream_t s = (cudaStream_t)stream;
    if (A->scalar_type == SPMM_F32) {
        if (index_type == SPMM_INDEX_I32)
            return boo_to_csr_impl<float, int32_t>(A, w, (int32_t *)indptr, (int32_t *)indices, (float *)values, s);
        return boo_to_csr_impl<float, int64_t>(A, w, (int64_t *)indptr, (int64_t *)indices, (float *)values, s);
    }
    if (index_type == SPMM_INDEX_I32)
        return boo_to_csr_impl<double, int32_t>(A, w, (int32_t *)indptr, (int32_t *)indices, (double *)values, s);
    return boo_to_csr_impl<double, int64_t>(A, w, (int64_t *)indptr, (int64_t *)indices, (double *)values, s);
}

extern "C" size_t spmm_pbr_to_csr_workspace_size(const spmm_pbr_dev *A) {
    if (!A || A->rows < 0) return 0;
    const size_t sb = A->scalar_type == SPMM_F64 ? 8 : 4;
    return conv_layout(A->rows, A->nnz_c + A->rem_nnz, sb, nullptr, 0, nullptr) + 256;
}

extern "C" int spmm_pbr_to_csr(const spmm_pbr_dev *A, void *indptr, void *indices, void *values, int index_type,
                               void *workspace, size_t workspace_bytes, spmm_stream_t stream) {
    if (!A || !indptr || A->rows < 0 || A->cols < 0 || A->block_rows < 1 || A->block_cols < 1 ||
        A->block_rows * A->block_cols > 64)
        return SPMM_EINVAL;
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return SPMM_EINVAL;
    if (A->index_type != SPMM_INDEX_I32 && A->index_type != SPMM_INDEX_I64) return SPMM_EINVAL;
    if (index_type != SPMM_INDEX_I32 && index_type != SPMM_INDEX_I64) return SPMM_EINVAL;
    const int64_t n = A->nnz_c + A->rem_nnz;
    if (n > 0xFFFFFFFFLL || A->rows > 0x7fffffffLL || A->cols > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    if (n > 0 && (!indices || !values)) return SPMM_EINVAL;
    if (!workspace || workspace_bytes < spmm_pbr_to_csr_workspace_size(A)) return SPMM_EWORKSPACE;
    ConvWs w;
    conv_layout(A->rows, n, A->scalar_type == SPMM_F64 ? 8 : 4, workspace, workspace_bytes, &w);
    cudaStream_t s = (cudaStream_t)stream;
    const bool pi64 = A->index_type == SPMM_INDEX_I64, oi64 = index_type == SPMM_INDEX_I64;
    if (A->scalar_type == SPMM_F32) {
        if (!pi64 && !oi64)
            return pbr_to_csr_impl<float, int32_t, int32_t>(A, w, (int32_t *)indptr, (int32_t *)indices,
                                                            (float *)values, s);
        if (!pi64 && oi64)
            return pbr_to_csr_impl<float, int64_t, int32_t>(A, w, (int64_t *)indptr, (int64_t *)indices,
                                                            (float *)values, s);
        if (pi64 && !oi64)
            return pbr_to_csr_impl<float, int32_t, int64_t>(A, w, (int32_t *)indptr, (int32_t *)indices,
                                                            (float *)values, s);
        return pbr_to_csr_impl<float, int64_t, int64_t>(A, w, (int64_t *)indptr, (int64_t *)indices,
                                                        (float *)values, s);
    }
    if (!pi64 && !oi64)
        return pbr_to_csr_impl<double, int32_t, int32_t>(A, w, (int32_t *)indptr, (int32_t *)indices,
                                                         (double *)values, s);
    if (!pi64 && oi64)
        return pbr_to_csr_impl<double, int64_t, int32_t>(A, w, (int64_t *)indptr, (int64_t *)indices,
                                                         (double *)values, s);
    if (pi64 && !oi64)
        return pbr_to_csr_impl<double, int32_t, int64_t>(A, w, (int32_t *)indptr, (int32_t *)indices,
                                                         (double *)values, s);
    return pbr_to_csr_impl<double, int64_t, int64_t>(A, w, (int64_t *)indptr, (int64_t *)indices,
                                                     (double *)values, s);
}
