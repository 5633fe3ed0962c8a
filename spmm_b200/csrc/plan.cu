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
//     load-balanced nnz-flat pass computes Y (plan.cuh: plan_row_view).
// The plan lives in a caller-owned device buffer; the product reads it
// through spmm_launch_cfg::plan.
#include "plan.cuh"

namespace spmm {
namespace {

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

}  // namespace
}  // namespace spmm

using namespace spmm;

extern "C" size_t spmm_boo_plan_size(const spmm_boo_dev *A) {
    if (!A || A->n_rg < 0 || A->rows < 0 || A->nb < 0) return 0;
    if (A->nb > 0x7fffffffLL) return 0;
    return plan_layout(A).total;
}

extern "C" size_t spmm_boo_plan_workspace_size(const spmm_boo_dev *A) {
    if (!A || A->rows < 0) return 0;
    return plan_layout(A).row_view ? spmm_boo_to_csr_workspace_size(A) : 0;
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
    if (L.row_view)
        return spmm_boo_to_csr(A, base + L.rv_ptr, base + L.rv_col, base + L.rv_val, SPMM_INDEX_I32, workspace,
                               workspace_bytes, stream);
    return SPMM_OK;
}
