// build_noalloc.cu -- BOO build for callers that cannot allocate device memory.
//
// Some callers of this library must not call cudaMalloc (or any allocator):
// code running inside a framework that owns every device allocation through
// its own pool, a real-time or safety-critical loop where an allocation can
// block or fail at an arbitrary moment, or a plugin host that forbids its
// plugins to grow the device heap.  spmm_boo_build_noalloc() serves them: it
// runs the same two builder phases as spmm_boo_build_analyze/_emit, but their
// scratch memory is a fixed array compiled into this file instead of a
// caller-provided workspace.
//
//  * The array is kNoallocScratchBytes (32 MiB) of device memory.  Every GPU on
//    which the library's module holding it is loaded keeps those 32 MiB until
//    the process exits.
//  * Problems whose workspace (spmm_boo_build_workspace_size) exceeds it are
//    rejected with SPMM_ESCRATCH before any device work -- about half a
//    million nonzeros for a square matrix.
//  * Host code cannot pass the array's name to a kernel: in host code the
//    name is a host-side shadow, not a device address.  So every call looks
//    the device address up on the current device with cudaGetSymbolAddress
//    (it allocates nothing) and hands that to the builder; nothing is cached,
//    so a call after a device reset or on another device needs no set-up.
//  * All calls share the array and it keeps the previous call's contents; the
//    builder initialises everything it reads.  Calls whose GPU work overlaps
//    (different streams or threads, same device) race on the array and must
//    be serialised by the caller.
#include "common.cuh"

namespace {

constexpr size_t kNoallocScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// Device address of the scratch array on the current device.
int scratch_address(void **addr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
        (void)cudaGetLastError();
        return SPMM_ECUDA;
    }
    *addr = p;
    return SPMM_OK;
}

}  // namespace

extern "C" int spmm_boo_build_noalloc(const spmm_csr_dev *A, const int32_t *row_labels,
                                      const int32_t *col_labels, int policy, int64_t threshold,
                                      int nz_order, spmm_boo_dev *out, spmm_stream_t stream) {
    if (!A || !out) return SPMM_EINVAL;
    if (A->rows < 0 || A->cols < 0 || A->nnz < 0) return SPMM_EINVAL;
    const size_t need = spmm_boo_build_workspace_size(A->rows, A->cols, A->nnz);
    if (need == 0 || need > kNoallocScratchBytes) return SPMM_ESCRATCH;
    void *scratch = nullptr;
    SPMM_TRY(scratch_address(&scratch));
    spmm_boo_dev sizes = *out;
    SPMM_TRY(spmm_boo_build_analyze(A, row_labels, col_labels, policy, threshold, nz_order, scratch,
                                    kNoallocScratchBytes, &sizes, stream));
    // the caller's arrays were sized for the worst case; record the real sizes
    out->rows = sizes.rows;
    out->cols = sizes.cols;
    out->total_nnz = sizes.total_nnz;
    out->n_rg = sizes.n_rg;
    out->n_cg = sizes.n_cg;
    out->nb = sizes.nb;
    out->nnz_c = sizes.nnz_c;
    out->rem_nnz = sizes.rem_nnz;
    out->tail_nnz = sizes.tail_nnz;
    out->max_nr = sizes.max_nr;
    out->max_nc = sizes.max_nc;
    out->max_nnz_blk = sizes.max_nnz_blk;
    out->nz_order = sizes.nz_order;
    out->scalar_type = sizes.scalar_type;
    return spmm_boo_build_emit(A, row_labels, col_labels, policy, threshold, nz_order, scratch,
                               kNoallocScratchBytes, out, stream);
}
