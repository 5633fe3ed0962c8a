/*
 * spmm_b200.h -- C ABI of the B200 (sm_100a) BOO / PBR SpMM engine.
 *
 * Drop-in boundary for the hot path of Dayan135/SPMM (torch_fast_spdmm):
 * GPU format construction (csr_to_boo, csr_to_pbr) and Y = A*X with A in the
 * BOO or PBR format.  Every entry point takes plain device pointers and sizes
 * and a CUDA stream; no torch types cross this boundary.
 *
 * Conventions
 *   - Ownership: the caller owns every buffer (inputs, outputs, workspace).
 *     Device memory the library allocates itself, all of it named here:
 *       * spmm_hem_labels / spmm_hem_hierarchy take their per-level scratch
 *         from the device's default stream-ordered pool (cudaMallocAsync /
 *         cudaFreeAsync) and release it before returning; while they run the
 *         pool's release threshold is raised so freed scratch stays mapped
 *         between levels, and on return the threshold is restored and the
 *         pool trimmed to it (other users of that pool see the raised
 *         threshold meanwhile);
 *       * spmm_boo_build_noalloc uses a fixed 32 MiB array compiled into the
 *         library (one per device that loads it, held until exit);
 *     the builders, products and conversions allocate nothing: their scratch
 *     is the caller's workspace (*_workspace_size()), and a product given too
 *     little returns SPMM_EWORKSPACE.
 *   - Errors: every entry point returns an int status (SPMM_OK == 0).  No C++
 *     exception crosses the ABI.  spmm_status_string() gives the text.
 *     Device-side outcomes of an asynchronous product (a bounded wait that
 *     expired: SPMM_ETIMEOUT) land in the call's status word
 *     (spmm_launch_cfg::status); a call given none reports into one
 *     process-wide word shared by all such calls, read by spmm_tc_status().
 *   - Streams: work is enqueued on `stream` (cudaStream_t; NULL = legacy
 *     default stream) in order with the caller's other work on that stream.
 *     The *_analyze builder phases, spmm_boo_build_noalloc, spmm_pbr_to_csr
 *     and the HEM labellers block the host (they return sizes or check data).
 *   - Threading: re-entrant; concurrent calls on different streams with
 *     different buffers (workspaces and status words included) are safe.
 *     Process-wide state: the fallback status word above, the noalloc
 *     scratch (overlapping noalloc calls race on it) and the product-launch
 *     counter (spmm_product_launches(), a measurement aid).
 *   - Devices: work runs on the CUDA device current on the calling thread; all
 *     pointers must belong to that device.
 *   - Dense operands: X is [batch][cols][K] and Y is [batch][rows][K], both
 *     C-contiguous in the format's scalar type.  Y is fully overwritten.
 */
#ifndef SPMM_B200_H
#define SPMM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *spmm_stream_t; /* == cudaStream_t */

enum spmm_status {
    SPMM_OK = 0,
    SPMM_EINVAL = 1,          /* bad argument (policy, order, sizes, null pointer) */
    SPMM_ELABEL = 2,          /* cluster label out of range */
    SPMM_EOVERFLOW_U16 = 3,   /* a kept BOO block's local index space exceeds uint16 */
    SPMM_EDUPLICATE = 4,      /* PBR input has duplicate (row, col) entries */
    SPMM_ECUDA = 5,           /* a CUDA runtime call or kernel launch failed */
    SPMM_EWORKSPACE = 6,      /* workspace smaller than *_workspace_size() asked for */
    SPMM_EUNSUPPORTED = 7,    /* size or type outside what this build handles */
    SPMM_EALIGN = 8,          /* a pointer lacks the alignment its dtype requires */
    SPMM_ESCRATCH = 9,        /* problem larger than spmm_boo_build_noalloc's fixed scratch */
    SPMM_ETIMEOUT = 10,       /* a bounded device wait expired (in a status word; Y incomplete) */
    SPMM_ENCCL = 11           /* a collective failed (the multi-GPU helpers above this ABI) */
};

enum spmm_index_type { SPMM_INDEX_I32 = 0, SPMM_INDEX_I64 = 1 };
enum spmm_scalar_type { SPMM_F32 = 0, SPMM_F64 = 1 };
enum spmm_boo_policy { SPMM_BOO_KEEP = 0, SPMM_BOO_MERGE = 1, SPMM_BOO_REMAINDER = 2,
                       SPMM_BOO_TAIL_BATCH = 3 };
enum spmm_boo_order { SPMM_BOO_ROWMAJOR = 0, SPMM_BOO_COLMAJOR = 1 };

/* A CSR matrix in device memory. */
typedef struct {
    int64_t rows, cols, nnz;
    const void *indptr;   /* rows+1 entries of index_type */
    const void *indices;  /* nnz entries of index_type */
    const void *values;   /* nnz entries of scalar_type */
    int32_t index_type;   /* enum spmm_index_type */
    int32_t scalar_type;  /* enum spmm_scalar_type */
} spmm_csr_dev;

/*
 * BOO (Blocked COO) in device memory.  Field meanings follow the reference's
 * boo_matrix_t (torch_fast_spdmm/boo_matrix/boo_matrix.hpp:56-138); index
 * arrays are int32 and nz_idx is uint16, as the reference stages them onto the
 * GPU (torch_fast_spdmm/torch_fast_spdmm/boo.py:54-96).
 */
typedef struct {
    int64_t rows, cols, total_nnz;
    int64_t n_rg, n_cg;            /* row / column groups */
    int64_t nb, nnz_c;             /* blocks, nonzeros stored in blocks */
    int64_t rem_nnz, tail_nnz;     /* CSR remainder, flat COO tail */
    int64_t max_nr, max_nc, max_nnz_blk;
    int32_t nz_order;              /* enum spmm_boo_order */
    int32_t scalar_type;           /* enum spmm_scalar_type */
    int32_t *row_grp_ptr;          /* n_rg+1 */
    int32_t *row_ids;              /* rows */
    int32_t *col_grp_ptr;          /* n_cg+1 */
    int32_t *col_ids;              /* cols */
    int32_t *blk_row_grp;          /* nb, ascending (blocks sorted by (rg, cg)) */
    int32_t *blk_col_grp;          /* nb */
    int32_t *blk_nz_ptr;           /* nb+1 */
    uint8_t *blk_shift;            /* nb */
    uint16_t *nz_idx;              /* nnz_c: (local_row << shift) | local_col */
    void *nz_val;                  /* nnz_c */
    int32_t *rem_indptr;           /* rows+1 */
    int32_t *rem_col_ind;          /* rem_nnz */
    void *rem_vals;                /* rem_nnz */
    int32_t *tail_row;             /* tail_nnz, non-decreasing (CSR traversal order) */
    int32_t *tail_col;             /* tail_nnz */
    void *tail_val;                /* tail_nnz */
} spmm_boo_dev;

/*
 * PBR (packed 64-bit-bitset blocks) in device memory.  Field meanings follow
 * the reference's pbr_matrix_t (torch_fast_spdmm/pbr_matrix/pbr_matrix.hpp:
 * 98-167) as staged by PBRMatrix.to() (torch_fast_spdmm/torch_fast_spdmm/
 * __init__.py:17-40): codes as 64-bit words, coordinates, offsets and the
 * remainder in the host index type.  Blocks are grouped by stripe
 * (row / block_rows) in ascending stripe order; the builder here emits them in
 * (stripe, block column) order.
 */
typedef struct {
    int64_t rows, cols, block_rows, block_cols, total_nnz;
    int64_t nb, nnz_c, rem_nnz;
    int32_t index_type;            /* enum spmm_index_type (coords, offsets, remainder) */
    int32_t scalar_type;
    uint64_t *codes;               /* nb: bit (r*block_cols + c) set for a nonzero */
    void *coords;                  /* 2*nb: top-left (row, col) of each block */
    void *offsets;                 /* nb+1: start of each block's values in data */
    void *data;                    /* nnz_c: values, consumed in bit order */
    void *rem_indptr;              /* rows+1 */
    void *rem_col_ind;             /* rem_nnz */
    void *rem_vals;                /* rem_nnz */
} spmm_pbr_dev;

/* Optional per-call settings; NULL selects the defaults.  No process-wide
 * tuning state: the reference's global setters (torch_fast_spdmm/kernels/
 * boo_kernel.cu:58-99) have no counterpart here. */
typedef struct {
    int32_t version;        /* 1, or 2 (adds `status`) */
    int32_t slab_features;  /* remainder-major BOO products: 0 = automatic (default): half a
                             * warp per row for a remainder of <= 16 entries per row on
                             * average with K <= 64 float32 / 32 float64 (no workspace),
                             * else the nnz-flat chunks with X rows staged by asynchronous
                             * copies; > 0 = the nnz-flat chunks; < 0 = rows through
                             * registers (no workspace) */
    int32_t engine;         /* enum spmm_engine (BOO product only; PBR ignores it) */
    int32_t wait_us;        /* bounded device waits of the tensor-core product: 0 = about
                             * 2 s (default); > 0 = give up after about this many
                             * microseconds (tests of the timeout path) */
    void *workspace;        /* device scratch of the BOO product, 16-byte aligned: at least */
    uint64_t workspace_bytes; /* spmm_boo_matmul_workspace_size() bytes when that is > 0 */
    int32_t *status;        /* version 2, optional: a device int32 the call sets to 0
                             * (stream-ordered) and a kernel sets to SPMM_ETIMEOUT when one
                             * of its bounded waits expired; read it after the stream */
    int32_t flags;          /* version 2: 0, or SPMM_CFG_EXPIRE_FIRST_WAIT */
    int32_t reserved;       /* version 2: 0 */
    const void *plan;       /* version 2, optional: this matrix's product plan
                             * (spmm_boo_plan_build), or NULL */
} spmm_launch_cfg;

/* spmm_launch_cfg::flags.  SPMM_CFG_EXPIRE_FIRST_WAIT (tests of the timeout
 * path; needs wait_us > 0): every tensor-core worker's first bounded wait is
 * on a barrier nothing arrives on, so it expires after wait_us, the launch
 * stops early (Y incomplete) and the status word reads SPMM_ETIMEOUT. */
enum spmm_cfg_flags { SPMM_CFG_EXPIRE_FIRST_WAIT = 1 };

/* Which units multiply the BOO blocks.  AUTO takes the tensor cores when the
 * matrix is float32, K is a multiple of 128 and every block fits 64 x 64
 * (3xTF32 split: within the float32 tolerance), else the CUDA cores. */
enum spmm_engine {
    SPMM_ENGINE_AUTO = 0,
    SPMM_ENGINE_CUDA_CORES = 1,   /* fp32/fp64 FMA, the reference CPU path's summation order */
    SPMM_ENGINE_TENSOR_CORES = 2, /* tcgen05 3xTF32; SPMM_EUNSUPPORTED when not applicable */
    SPMM_ENGINE_TENSOR_CORES_TF32 = 3  /* opt-in: one tf32 product per K step (tf32 accuracy,
                                        * about 2e-3 relative; never chosen by AUTO) */
};

/* ---- status ---------------------------------------------------------- */
const char *spmm_status_string(int status);
int spmm_abi_version(void);

/* ---- BOO build (replaces csr_to_boo, torch_fast_spdmm/boo_matrix/
 * boo_matrix.cpp:53-274, bound at bindings/bindings.cpp:210-213) ---------
 *
 * Two phases over one caller-owned workspace:
 *   1. spmm_boo_build_analyze() runs the whole build up to the output sizes and
 *      fills the size fields of *sizes (rows, cols, total_nnz, n_rg, n_cg, nb,
 *      nnz_c, rem_nnz, tail_nnz, max_nr, max_nc, max_nnz_blk, nz_order,
 *      scalar_type).  It blocks the host until the sizes are known.
 *   2. The caller allocates the arrays of a spmm_boo_dev with those sizes and
 *      calls spmm_boo_build_emit() with the same arguments and workspace,
 *      untouched in between.  Emit is asynchronous on `stream`.
 * Labels are int32 device arrays of length rows / cols with values in
 * [0, rows) / [0, cols); the number of groups is max(label) + 1.
 */
size_t spmm_boo_build_workspace_size(int64_t rows, int64_t cols, int64_t nnz);
int spmm_boo_build_analyze(const spmm_csr_dev *A, const int32_t *row_labels,
                           const int32_t *col_labels, int policy, int64_t threshold,
                           int nz_order, void *workspace, size_t workspace_bytes,
                           spmm_boo_dev *sizes, spmm_stream_t stream);
int spmm_boo_build_emit(const spmm_csr_dev *A, const int32_t *row_labels,
                        const int32_t *col_labels, int policy, int64_t threshold, int nz_order,
                        void *workspace, size_t workspace_bytes, spmm_boo_dev *out,
                        spmm_stream_t stream);

/* ---- BOO build without any device allocation --------------------------
 * No counterpart in the reference: for callers that cannot allocate device
 * memory (a framework that owns all device memory through its own pool, a
 * loop where an allocation may block or fail, a plugin host that forbids heap
 * growth).  One call runs both builder phases with their scratch in a fixed
 * 32 MiB device array compiled into the library instead of a caller
 * workspace; nothing is allocated.  Problems whose
 * spmm_boo_build_workspace_size() exceeds 32 MiB (about half a million
 * nonzeros) return SPMM_ESCRATCH before any device work.
 *   - `out` arrays are caller-allocated for the worst case: row_grp_ptr and
 *     rem_indptr rows+1, row_ids rows, col_grp_ptr cols+1, col_ids cols,
 *     blk_nz_ptr nnz+1, every other array nnz entries.  On return the size
 *     fields of *out hold the real sizes.
 *   - Each call looks up the array's device address on the current device
 *     (cudaGetSymbolAddress; no allocation).
 *   - Blocks the host until the sizes are known, like the analyze phase.
 *   - All calls share the array: calls whose GPU work overlaps race and must
 *     be serialised by the caller. */
int spmm_boo_build_noalloc(const spmm_csr_dev *A, const int32_t *row_labels,
                           const int32_t *col_labels, int policy, int64_t threshold, int nz_order,
                           spmm_boo_dev *out, spmm_stream_t stream);

/* ---- PBR build (replaces csr_to_pbr, torch_fast_spdmm/pbr_matrix/
 * pbr_matrix.cpp:333-448, bound at bindings/bindings.cpp:180-183) ---------
 * Same two-phase protocol.  block_rows * block_cols <= 64.  Keeps a block iff
 * popcount(code) >= min_nnz_per_block (the reference's uint8_t parameter,
 * pbr_matrix.cpp:398).  out->index_type selects the emitted index type. */
size_t spmm_pbr_build_workspace_size(int64_t rows, int64_t cols, int64_t nnz);
int spmm_pbr_build_analyze(const spmm_csr_dev *A, int64_t block_rows, int64_t block_cols,
                           int min_nnz_per_block, void *workspace, size_t workspace_bytes,
                           spmm_pbr_dev *sizes, spmm_stream_t stream);
int spmm_pbr_build_emit(const spmm_csr_dev *A, int64_t block_rows, int64_t block_cols,
                        int min_nnz_per_block, void *workspace, size_t workspace_bytes,
                        spmm_pbr_dev *out, spmm_stream_t stream);

/* ---- SpMM ------------------------------------------------------------ */

/* Y = A*X for a BOO matrix (replaces boo_spmm_cuda_impl / boo_run_into,
 * torch_fast_spdmm/bindings/bindings_boo.cu:34-313, bound as
 * boo_spmm_cuda_{f32,f64} at bindings_boo.cu:408-476).  Blocks, CSR
 * remainder and COO tail of a row group are summed by the CTA (or tensor-core
 * worker) that owns the group and every Y element is written once, with no
 * memset and no atomics: one launch on CUDA cores, two on the tensor cores
 * (X gathered by column group, then the product), four for remainder-major
 * matrices (the nnz-flat remainder's plan, chunks and fix-up, then blocks and
 * tail added by the block kernel). */
int spmm_boo_matmul(const spmm_boo_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                    const spmm_launch_cfg *cfg, spmm_stream_t stream);

/* The same product restricted to row groups [rg_begin, rg_end): exactly the Y
 * rows of those groups (row_ids[row_grp_ptr[rg_begin] .. row_grp_ptr[rg_end]))
 * are written, and only the X rows their blocks, remainder and tail entries
 * use are read, so a caller can multiply row groups as soon as their X rows
 * have arrived and copy their Y rows out while later groups run (no
 * reference counterpart; the reference has no partial product).  Same
 * configuration and workspace as spmm_boo_matmul.  SPMM_EUNSUPPORTED for
 * remainder-major matrices (CSR remainder >= half of the nonzeros) unless
 * the range is the whole matrix. */
int spmm_boo_matmul_groups(const spmm_boo_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                           int64_t rg_begin, int64_t rg_end, const spmm_launch_cfg *cfg, spmm_stream_t stream);

/* ---- BOO product plan (replaces the reference's execution plans,
 * torch_fast_spdmm/torch_fast_spdmm/boo_plan.py:11-123, which precompute
 * launch tables once per matrix) --------------------------------------------
 * Per-matrix tables the product reads through spmm_launch_cfg::plan instead
 * of recomputing them every call: the first block of every row group, and
 * for remainder-major matrices whose blocks and tail hold at least 1/64 of the
 * entries, a row-ordered copy of every entry that one load-balanced pass
 * multiplies (the layout follows from A's size fields).  The plan is a
 * caller-owned device buffer of spmm_boo_plan_size() bytes, 256-byte
 * aligned; building it takes spmm_boo_plan_workspace_size() bytes of scratch
 * (0 when no row-ordered copy is made).  A plan stays valid while the
 * matrix's arrays are unchanged; it must not be used with another matrix. */
size_t spmm_boo_plan_size(const spmm_boo_dev *A);
size_t spmm_boo_plan_workspace_size(const spmm_boo_dev *A);
int spmm_boo_plan_build(const spmm_boo_dev *A, void *plan, size_t plan_bytes, void *workspace,
                        size_t workspace_bytes, spmm_stream_t stream);

/* Bytes of device scratch the BOO product needs in cfg->workspace for these
 * operands and settings: the X panels gathered by column group (tensor-core
 * product) or the chunk table and partial rows of the nnz-flat remainder
 * (remainder-major matrices); 0 when none is needed.  spmm_boo_matmul
 * returns SPMM_EWORKSPACE when it is needed and missing. */
size_t spmm_boo_matmul_workspace_size(const spmm_boo_dev *A, int64_t batch, int64_t K,
                                      const spmm_launch_cfg *cfg);

/* The process-wide status word of products called without one
 * (spmm_launch_cfg::status == NULL; no reference counterpart): 0, or
 * SPMM_ETIMEOUT once a bounded wait of such a call expired.  Synchronises the
 * device; `clear` resets the word.  Returns -1 when the CUDA runtime fails. */
int spmm_tc_status(int clear);

/* Product kernels (BOO and PBR SpMM, the tensor-core gather pass included)
 * this library has launched since it was loaded, counted on the host after
 * each successful launch (no reference counterpart; a measurement aid). */
uint64_t spmm_product_launches(void);

/* Y = A*X for a PBR matrix (replaces pbr_spmm_cuda_dispatch / pbr_run_into,
 * torch_fast_spdmm/bindings/bindings_kernels.cu:18-123, bound as
 * pbr_spmm_cuda_{i32,i64}_{f32,f64} at bindings_kernels.cu:433-459).  Any
 * block shape with block_rows * block_cols <= 64 and any K. */
int spmm_pbr_matmul(const spmm_pbr_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                    const spmm_launch_cfg *cfg, spmm_stream_t stream);

/* CSR from a BOO matrix on the GPU (replaces boo_to_csr, torch_fast_spdmm/
 * boo_matrix/boo_matrix.cpp:277-333, bound at bindings/bindings.cpp): every
 * stored entry -- blocks, CSR remainder, COO tail -- with each row ordered by
 * (column, value) like the reference's per-row sort of (column, value) pairs.
 * indptr (rows+1), indices and values (nnz_c + rem_nnz + tail_nnz) are
 * caller-allocated; index_type (enum spmm_index_type) is the output index
 * type.  Scratch: spmm_boo_to_csr_workspace_size() bytes. */
size_t spmm_boo_to_csr_workspace_size(const spmm_boo_dev *A);
int spmm_boo_to_csr(const spmm_boo_dev *A, void *indptr, void *indices, void *values, int index_type,
                    void *workspace, size_t workspace_bytes, spmm_stream_t stream);

/* CSR from a PBR matrix on the GPU (replaces pbr_to_csr, torch_fast_spdmm/
 * pbr_matrix/pbr_matrix.cpp:279-331): block values in bit order, then the
 * remainder, each row ordered by (column, value).  SPMM_EINVAL when a block
 * bit lies past the last row (the reference's RuntimeError); synchronises the
 * stream to check that.  Outputs and scratch as for spmm_boo_to_csr. */
size_t spmm_pbr_to_csr_workspace_size(const spmm_pbr_dev *A);
int spmm_pbr_to_csr(const spmm_pbr_dev *A, void *indptr, void *indices, void *values, int index_type,
                    void *workspace, size_t workspace_bytes, spmm_stream_t stream);

/* Multilevel heavy-edge matching labels on the GPU (replaces the host HEM of
 * torch_fast_spdmm/torch_fast_spdmm/clustering.py:128-351, cluster='hem'):
 * one label per row of the binary pattern (indptr int64 rows+1, indices int32,
 * canonical: sorted, no duplicates), equal to the reference algorithm's
 * labels before its cap enforcement.  Columns of degree > hub_degree are
 * ignored, each row keeps its topk heaviest similarity edges (topk < 0: all),
 * max_size / max_nnz < 0 mean no cap.  labels: rows int64 (device).  Scratch
 * from the stream-ordered allocator; synchronises the stream. */
int spmm_hem_labels(int64_t rows, int64_t cols, const int64_t *indptr, const int32_t *indices, int64_t target,
                    int64_t max_size, int64_t max_nnz, int64_t hub_degree, int64_t topk, int32_t residual_rounds,
                    int32_t feasible_first, int64_t *labels, spmm_stream_t stream);

/* The same labels, plus the matching hierarchy (replaces the `hierarchy`
 * record of the reference's _hem_labels, clustering.py:271-282, behind
 * cluster_axis(..., hem_hierarchy=[])): levels (device, level_slots x rows
 * int64, level_slots >= spmm_hem_level_slots(target)) receives the identity
 * labels, then the labels after each level that matched, finest to coarsest;
 * *n_levels (host) the number of arrays written.  levels may be NULL. */
int64_t spmm_hem_level_slots(int64_t target);
int spmm_hem_hierarchy(int64_t rows, int64_t cols, const int64_t *indptr, const int32_t *indices, int64_t target,
                       int64_t max_size, int64_t max_nnz, int64_t hub_degree, int64_t topk, int32_t residual_rounds,
                       int32_t feasible_first, int64_t *labels, int64_t *levels, int64_t level_slots,
                       int64_t *n_levels, spmm_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SPMM_B200_H */
