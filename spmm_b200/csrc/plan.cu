// plan.cu -- per-matrix product plans for the BOO product.
//
// The reference prepares execution plans for its launches once per matrix
// (torch_fast_spdmm/torch_fast_spdmm/boo_plan.py:11-123: size-class buckets
// and precomputed row tables).  The tables the products here can reuse are
// different ones:
//   * the first block of every row group, so a CTA or tensor-core worker
//     reads its group's block range with one load instead of a search over
//     the block list;
//   * for remainder-major matrices with scattered blocks, a row-ordered copy
//     of every stored entry (the CSR view spmm_boo_to_csr produces), so one
//     load-balanced nnz-flat pass computes Y (plan.cuh: plan_row_view_rem);
//   * for tensor-core matrices, whether the column order is the identity
//     (64-column panels are then read straight from X, not from a gathered
//     copy);
//   * the same copy for matrices of a few entries per row, multiplied a warp
//     per row (plan.cuh: plan_short_rows), with a flag telling whether the
//     row-group order is the identity (the product then skips row_ids).
// The plan lives in a caller-owned device buffer; the product reads it
// through spmm_launch_cfg::plan.
#include "plan.cuh"

namespace spmm {
namespace {

__global__ void fill_i32_kernel(int32_t *__restrict__ out, int64_t n, int32_t v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = v;
}

// *flag = 0 when some position k holds another row than k (the flag starts at 1).
__global__ void ident_kernel(const int32_t *__restrict__ row_ids, int64_t rows, int32_t *__restrict__ flag) {
    bool same = true;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < rows; k += (int64_t)gridDim.x * blockDim.x)
        same &= row_ids[k] == k;
    if (!__all_sync(0xffffffffu, same) && (threadIdx.x & 31) == 0) *flag = 0;
}

// rg_blk[rg] = first block whose row group is >= rg, for rg in [0, n_rg].
__global__ void rg_blk_kernel(const int32_t *__restrict__ blk_row_grp, int64_t nb, int64_t n_rg,
                              int32_t *__restrict__ rg_blk) {
    for (int64_t rg = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; rg <= n_rg;
         rg += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = 0, hi = nb;
        while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if ((int64_t)__ldg(blk_row_grp + mid) < rg) lo = mid + 1; else hi = mid;
        }
        rg_blk[rg] = (int32_t)lo;
    }
}

// Packing choice per block: a sparse block (fewer than kDenseNnz entries)
// whose entries use at most two quads of its column group, with at least
// three entries per quad, is packed; nslot[b] = its quads (0 when not).
__global__ void pack_mark_kernel(const int32_t *__restrict__ blk_nz_ptr, const uint8_t *__restrict__ blk_shift,
                                 const uint16_t *__restrict__ nz_idx, int64_t nb, uint8_t *__restrict__ packed,
                                 uint16_t *__restrict__ qmask, int32_t *__restrict__ nslot) {
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
        const int32_t k0 = __ldg(blk_nz_ptr + b), k1 = __ldg(blk_nz_ptr + b + 1);
        const int n = k1 - k0;
        uint32_t m = 0;
        if (n < kDenseNnz) {
            const uint32_t cm = (1u << __ldg(blk_shift + b)) - 1u;
            for (int32_t k = k0; k < k1; ++k) m |= 1u << ((__ldg(nz_idx + k) & cm) >> 2);
        }
        const int q = __popc(m);
        const bool pk = n < kDenseNnz && q >= 1 && q <= 2 && n >= 3 * q;
        packed[b] = pk ? 1 : 0;
        qmask[b] = (uint16_t)(pk ? m : 0u);
        nslot[b] = pk ? q : 0;
    }
}

// Slots of the packed blocks at their scanned positions (quads ascending),
// and each row group's first slot (through its first block).
__global__ void pack_fill_kernel(const uint16_t *__restrict__ qmask, const int32_t *__restrict__ start, int64_t nb,
                                 const int32_t *__restrict__ rg_blk, int64_t n_rg, int32_t *__restrict__ slots,
                                 int32_t *__restrict__ rg_slot) {
    for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nb; b += (int64_t)gridDim.x * blockDim.x) {
        uint32_t m = qmask[b];
        int32_t at = start[b];
        while (m) {
            const int q = __ffs(m) - 1;
            m &= m - 1;
            slots[at++] = (int32_t)(b * 16 + q);
        }
    }
    for (int64_t rg = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; rg <= n_rg;
         rg += (int64_t)gridDim.x * blockDim.x)
        rg_slot[rg] = start[rg_blk[rg]];
}

// Scratch of the packing pass: per-block quad masks and slot counts (scanned
// in place), and the scan's partial sums.
inline size_t pack_workspace(int64_t nb) {
    return plan_align(2 * (size_t)nb) + plan_align(4 * (size_t)(nb + 1)) +
           plan_align(4 * (size_t)scan_temp_elems(nb + 1)) + 256;
}

}  // namespace
}  // namespace spmm

using namespace spmm;

extern "C" size_t spmm_boo_plan_size(const spmm_boo_dev *A) {
    if (!A || A->n_rg < 0 || A->rows < 0 || A->nb < 0) return 0;
    if (A->nb > 0x7fffffffLL) return 0;
    return plan_layout(A).total;
}

extern "C" size_t spmm_boo_plan_workspace_size(const spmm_boo_dev *A) {
    if (!A || A->rows < 0 || A->nb < 0) return 0;
    const PlanLayout L = plan_layout(A);
    size_t w = L.row_view ? spmm_boo_to_csr_workspace_size(A) : 0;
    if (L.packing) w = w > pack_workspace(A->nb) ? w : pack_workspace(A->nb);
    return w;
}

extern "C" int spmm_boo_plan_build(const spmm_boo_dev *A, void *plan, size_t plan_bytes, void *workspace,
                                   size_t workspace_bytes, spmm_stream_t stream) {
    if (!A || !plan || A->n_rg < 0 || A->rows < 0 || A->nb < 0) return SPMM_EINVAL;
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return SPMM_EINVAL;
    if (A->nb > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    if (A->nb && !A->blk_row_grp) return SPMM_EINVAL;
    if ((uintptr_t)plan & 255) return SPMM_EALIGN;
    const PlanLayout L = plan_layout(A);
    if (plan_bytes < L.total) return SPMM_EWORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t *base = static_cast<uint8_t *>(plan);
    const int64_t n = A->n_rg + 1;
    rg_blk_kernel<<<grid_for(n, 256), 256, 0, s>>>(A->blk_row_grp, A->nb, A->n_rg,
                                                   reinterpret_cast<int32_t *>(base + L.rg_blk));
    SPMM_LAUNCH_CHECK();
    if (L.packing) {
        if (!A->blk_nz_ptr || !A->blk_shift || !A->nz_idx) return SPMM_EINVAL;
        if (!workspace || workspace_bytes < pack_workspace(A->nb)) return SPMM_EWORKSPACE;
        uint8_t *wsp = static_cast<uint8_t *>(workspace);
        uint16_t *qmask = reinterpret_cast<uint16_t *>(wsp);
        int32_t *count = reinterpret_cast<int32_t *>(wsp + plan_align(2 * (size_t)A->nb));
        int32_t *temp = reinterpret_cast<int32_t *>(wsp + plan_align(2 * (size_t)A->nb) +
                                                    plan_align(4 * (size_t)(A->nb + 1)));
        const unsigned g = grid_for(A->nb, 256);
        pack_mark_kernel<<<g, 256, 0, s>>>(A->blk_nz_ptr, A->blk_shift, A->nz_idx, A->nb, base + L.packed, qmask,
                                          count);
        SPMM_LAUNCH_CHECK();
        SPMM_CUDA_TRY(cudaMemsetAsync(count + A->nb, 0, sizeof(int32_t), s));
        SPMM_TRY(exclusive_scan<int32_t>(count, count, A->nb + 1, temp, nullptr, s));
        pack_fill_kernel<<<grid_for(A->nb > A->n_rg + 1 ? A->nb : A->n_rg + 1, 256), 256, 0, s>>>(
            qmask, count, A->nb, reinterpret_cast<const int32_t *>(base + L.rg_blk), A->n_rg,
            reinterpret_cast<int32_t *>(base + L.slots), reinterpret_cast<int32_t *>(base + L.rg_slot));
        SPMM_LAUNCH_CHECK();
        if (A->cols && !A->col_ids) return SPMM_EINVAL;
        int32_t *cflag = reinterpret_cast<int32_t *>(base + L.cg_ident);
        fill_i32_kernel<<<1, 32, 0, s>>>(cflag, 1, 1);
        SPMM_LAUNCH_CHECK();
        if (A->cols) {
            ident_kernel<<<grid_for(A->cols, 256), 256, 0, s>>>(A->col_ids, A->cols, cflag);
            SPMM_LAUNCH_CHECK();
        }
    }
    if (L.short_rows) {
        if (!A->row_ids) return SPMM_EINVAL;
        int32_t *flag = reinterpret_cast<int32_t *>(base + L.rv_ident);
        fill_i32_kernel<<<1, 32, 0, s>>>(flag, 1, 1);
        SPMM_LAUNCH_CHECK();
        ident_kernel<<<grid_for(A->rows, 256), 256, 0, s>>>(A->row_ids, A->rows, flag);
        SPMM_LAUNCH_CHECK();
    }
    if (L.row_view)
        return spmm_boo_to_csr(A, base + L.rv_ptr, base + L.rv_col, base + L.rv_val, SPMM_INDEX_I32, workspace,
                               workspace_bytes, stream);
    return SPMM_OK;
}
