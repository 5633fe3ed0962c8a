// spmm_boo.cu -- Y = A*X for A in BOO format on sm_100a.
//
// Replaces the reference's block kernel + CSR-remainder kernel + tail kernel
// trio and their 3-stream fork/join over a memset Y (torch_fast_spdmm/
// bindings/bindings_boo.cu:34-118, kernels/boo_kernel.cu:410-595 and 905-937,
// kernels/pbr_kernel.cu:976-1049) with ONE launch in which a CTA owns a
// (row group, feature slab, batch) work item:
//   * blocks of the row group are contiguous (sorted by (rg, cg),
//     boo_matrix.cpp:123-125); the CTA stages their nonzeros in shared memory
//     as (global column, value) pairs in batches, with a per-row start table;
//   * each group of LPR lanes owns rows of the group and accumulates, in
//     registers, the row's block entries, then its CSR-remainder row, then its
//     tail entries (tail rows are non-decreasing: binary search);
//   * every Y element is stored exactly once -- no memset, no atomics.
// Per output row the nonzeros are summed in the reference CPU path's order
// (blocks in order, entries in order, remainder, tail; boo_matrix.cpp:
// 336-396), with fused multiply-adds.
#include <climits>

#include "plan.cuh"
#include "ptx.cuh"
#include "spmm_common.cuh"

namespace spmm {

int boo_matmul_tc(const spmm_boo_dev *A, const float *X, float *Y, int64_t batch, int64_t K, int64_t rg_first,
                  int64_t rg_end, void *ws, size_t ws_bytes, int32_t *status, int32_t wait_us, int32_t flags,
                  bool tf32_only, const uint8_t *plan, cudaStream_t s);
size_t boo_tc_workspace(const spmm_boo_dev *A, int64_t batch, int64_t K);

namespace {

constexpr int kBooThreads = 256;
constexpr int kRowsChunk = 32;      // rows of a row group handled per pass
constexpr int kStageCap = 2048;     // staged nonzeros per batch
constexpr int kMaxSeg = 32;         // block segments per batch (one per warp-0 lane)

template <typename S>
struct BooParams {
    int64_t rows, cols, K, batch, nb, tail_nnz;
    const int32_t *row_grp_ptr, *row_ids, *col_grp_ptr, *col_ids;
    const int32_t *blk_row_grp, *blk_col_grp, *blk_nz_ptr;
    const uint8_t *blk_shift;
    const uint16_t *nz_idx;
    const S *nz_val;
    const int32_t *rem_indptr, *rem_col;
    const S *rem_val;
    const int32_t *tail_row, *tail_col;
    const S *tail_val;
    const S *X;
    S *Y;
    int rowmajor;
    int skip_rem;   // remainder-major: Y already holds the CSR remainder (load-balanced
                    // kernels ran first); add blocks and tail to it, skip other groups
    // nnz-flat remainder: chunks of `chunk` entries, the row holding each
    // chunk's first entry, two partial-sum rows per (batch, chunk)
    int64_t rem_nnz, nch;
    int64_t n_rg, rgs_per_cta;   // block kernel: CTA x takes row groups rg_first + [x * rgs_per_cta, ...)
    int64_t rg_first;            //   up to n_rg (the end of the range, exclusive)
    const int32_t *rg_blk;       // plan: first block of every row group (null: search blk_row_grp)
    int32_t chunk;
    int32_t *chunk_row;
    S *part;
};

// first index in a[0..n) with a[i] >= key (a ascending)
__device__ __forceinline__ int64_t lower_bound_i32(const int32_t *a, int64_t n, int64_t key) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        int64_t mid = (lo + hi) >> 1;
        if ((int64_t)a[mid] < key) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// last segment s in [0, nseg) with start[s] <= e
__device__ __forceinline__ int find_seg(const int32_t *start, int nseg, int e) {
    int lo = 0, hi = nseg - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (start[mid] <= e) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <typename S>
struct BooSmem {
    int32_t col[kStageCap];
    S val[kStageCap];
    uint16_t lrow[kStageCap];
    uint16_t rt[kMaxSeg][kRowsChunk + 1];   // row start table per segment
    int32_t seg_start[kMaxSeg + 1];         // staging offset of each segment
    int32_t seg_k0[kMaxSeg];
    int32_t seg_cbase[kMaxSeg];
    uint8_t seg_shift[kMaxSeg];
    int32_t nseg, total;
    int64_t blk_lo, blk_hi, next_blk, next_k;
};

// acc += a * X[c, lane's features]; `vm` masks slots past K.
template <typename S, int VEC, int VPT, int LPR, int U>
__device__ __forceinline__ void accumulate(Frag<S, VEC> (&acc)[VPT], const int32_t *cols,
                                           const S *vals, int64_t e0, int64_t e1, const S *xl,
                                           int64_t K, const bool (&vm)[VPT]) {
    constexpr int STR = LPR * VEC;
    int64_t e = e0;
    for (; e + U <= e1; e += U) {
        S a[U];
        Frag<S, VEC> x[U][VPT];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            a[u] = vals[e + u];
            const S *xr = xl + (int64_t)cols[e + u] * K;
#pragma unroll
            for (int v = 0; v < VPT; ++v)
                if (vm[v]) x[u][v] = ldg_frag<S, VEC>(xr + v * STR);
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int v = 0; v < VPT; ++v)
                if (vm[v])
#pragma unroll
                    for (int q = 0; q < VEC; ++q) acc[v].v[q] = fma(a[u], x[u][v].v[q], acc[v].v[q]);
    }
    for (; e < e1; ++e) {
        const S a = vals[e];
        const S *xr = xl + (int64_t)cols[e] * K;
#pragma unroll
        for (int v = 0; v < VPT; ++v)
            if (vm[v]) {
                Frag<S, VEC> x = ldg_frag<S, VEC>(xr + v * STR);
#pragma unroll
                for (int q = 0; q < VEC; ++q) acc[v].v[q] = fma(a, x.v[q], acc[v].v[q]);
            }
    }
}

template <typename S, int VEC, int VPT, int LPR>
__global__ void __launch_bounds__(kBooThreads, VPT == 1 ? 4 : 1)
boo_spmm_kernel(const BooParams<S> p) {
    constexpr int NG = kBooThreads / LPR;        // lane groups per CTA
    constexpr int RPG = kRowsChunk / NG;          // rows per lane group per chunk
    constexpr int SLAB = LPR * VPT * VEC;
    constexpr int U = VPT == 1 ? 4 : 2;
    static_assert(RPG >= 1 && RPG * NG == kRowsChunk, "row mapping");
    __shared__ BooSmem<S> sm;

    const int tid = threadIdx.x;
    const int g = tid / LPR, l = tid % LPR;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t f0 = (int64_t)blockIdx.y * SLAB + (int64_t)l * VEC;
    bool vm[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) vm[v] = f0 + (int64_t)v * LPR * VEC < p.K;

    // row groups [rg_begin, rg_end); blocks found by one search, then walked
    const int64_t rg_begin = p.rg_first + (int64_t)blockIdx.x * p.rgs_per_cta;
    const int64_t rg_end = rg_begin + p.rgs_per_cta < p.n_rg ? rg_begin + p.rgs_per_cta : p.n_rg;
    if (warp == 0 && !p.rg_blk) {   // 32-way searches by warp 0 (no plan)
        const int64_t lo0 = warp_lower_bound(p.blk_row_grp, p.nb, rg_begin, lane);
        if (lane == 0) sm.blk_hi = lo0;
    }
    for (int64_t rg = rg_begin; rg < rg_end; ++rg) {
    __syncthreads();   // the previous group's readers of sm are done
    if (warp == 0) {
        int64_t lo, hi;
        if (p.rg_blk) {             // the plan's table
            lo = __ldg(p.rg_blk + rg);
            hi = __ldg(p.rg_blk + rg + 1);
        } else {
            lo = sm.blk_hi;
            hi = group_end(p.blk_row_grp, p.nb, lo, rg, lane);
        }
        if (lane == 0) {
            sm.blk_lo = lo;
            sm.blk_hi = hi;
        }
    }
    __syncthreads();
    const int64_t blk_lo = sm.blk_lo, blk_hi = sm.blk_hi;
    if (p.skip_rem && blk_lo == blk_hi && p.tail_nnz == 0) continue;   // nothing to add
    const int32_t rbase = p.row_grp_ptr[rg];
    const int32_t n_r = p.row_grp_ptr[rg + 1] - rbase;

    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K;
        for (int32_t r0 = 0; r0 < n_r; r0 += kRowsChunk) {
            const int R = n_r - r0 < kRowsChunk ? n_r - r0 : kRowsChunk;
            Frag<S, VEC> acc[RPG][VPT];
#pragma unroll
            for (int i = 0; i < RPG; ++i)
#pragma unroll
                for (int v = 0; v < VPT; ++v)
#pragma unroll
                    for (int q = 0; q < VEC; ++q) acc[i][v].v[q] = S(0);

            int64_t cur_blk = blk_lo;
            int64_t cur_k = blk_lo < blk_hi ? p.blk_nz_ptr[blk_lo] : 0;
            while (cur_blk < blk_hi) {
                // ---- plan a batch of block segments (warp 0) ----
                if (warp == 0) {
                    const int64_t b = cur_blk + lane;
                    const bool valid = b < blk_hi;
                    int64_t k0 = 0, k1 = 0;
                    if (valid) {
                        k0 = lane == 0 ? cur_k : (int64_t)p.blk_nz_ptr[b];
                        k1 = p.blk_nz_ptr[b + 1];
                    }
                    int64_t len = k1 - k0;
                    int64_t pre = len;  // inclusive prefix
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        int64_t n = __shfl_up_sync(kFullMask, pre, o);
                        if (lane >= o) pre += n;
                    }
                    const unsigned fits = __ballot_sync(kFullMask, valid && pre <= kStageCap);
                    const int nfit = __popc(fits);
                    if (nfit == 0) {
                        // first block alone overflows the stage: take a piece of it
                        if (lane == 0) {
                            sm.seg_start[0] = 0;
                            sm.seg_start[1] = kStageCap;
                            sm.seg_k0[0] = (int32_t)k0;
                            sm.seg_shift[0] = p.blk_shift[b];
                            sm.seg_cbase[0] = p.col_grp_ptr[p.blk_col_grp[b]];
                            sm.nseg = 1;
                            sm.total = kStageCap;
                            const int64_t nk = k0 + kStageCap;
                            sm.next_blk = nk >= k1 ? b + 1 : b;
                            sm.next_k = nk;
                        }
                    } else {
                        if (lane < nfit) {
                            sm.seg_start[lane] = (int32_t)(pre - len);
                            sm.seg_k0[lane] = (int32_t)k0;
                            sm.seg_shift[lane] = p.blk_shift[b];
                            sm.seg_cbase[lane] = p.col_grp_ptr[p.blk_col_grp[b]];
                        }
                        if (lane == nfit - 1) {
                            sm.seg_start[nfit] = (int32_t)pre;
                            sm.nseg = nfit;
                            sm.total = (int32_t)pre;
                            sm.next_blk = cur_blk + nfit;
                            sm.next_k = k1;  // == blk_nz_ptr[cur_blk + nfit]
                        }
                    }
                }
                __syncthreads();
                const int nseg = sm.nseg, total = sm.total;
                // ---- stage (global column, value, local row) ----
                for (int e = tid; e < total; e += kBooThreads) {
                    const int s = find_seg(sm.seg_start, nseg, e);
                    const int64_t k = (int64_t)sm.seg_k0[s] + (e - sm.seg_start[s]);
                    const uint32_t idx = p.nz_idx[k];
                    const uint32_t shift = sm.seg_shift[s];
                    sm.col[e] = p.col_ids[sm.seg_cbase[s] + (int32_t)(idx & ((1u << shift) - 1u))];
                    sm.val[e] = p.nz_val[k];
                    sm.lrow[e] = (uint16_t)(idx >> shift);
                }
                __syncthreads();
                if (p.rowmajor) {
                    // rt[s][q] = first staged entry of segment s with local row >= r0+q
                    for (int e = tid; e < total; e += kBooThreads) {
                        const int s = find_seg(sm.seg_start, nseg, e);
                        const int lr = sm.lrow[e];
                        const int prev = e == sm.seg_start[s] ? -1 : (int)sm.lrow[e - 1];
                        int qa = prev - r0 + 1, qb = lr - r0;
                        if (qa < 0) qa = 0;
                        if (qb > R) qb = R;
                        for (int q = qa; q <= qb; ++q) sm.rt[s][q] = (uint16_t)e;
                        if (e + 1 == sm.seg_start[s + 1]) {
                            int qc = lr - r0 + 1;
                            if (qc < 0) qc = 0;
                            for (int q = qc; q <= R; ++q) sm.rt[s][q] = (uint16_t)(e + 1);
                        }
                    }
                    __syncthreads();
                }
                // ---- accumulate ----
#pragma unroll
                for (int i = 0; i < RPG; ++i) {
                    const int q = g + i * NG;
                    if (q < R) {
                        for (int s = 0; s < nseg; ++s) {
                            if (p.rowmajor) {
                                accumulate<S, VEC, VPT, LPR, U>(acc[i], sm.col, sm.val, sm.rt[s][q],
                                                                sm.rt[s][q + 1], xl, p.K, vm);
                            } else {
                                const int lr = r0 + q;
                                for (int e = sm.seg_start[s]; e < sm.seg_start[s + 1]; ++e)
                                    if (sm.lrow[e] == lr)
                                        accumulate<S, VEC, VPT, LPR, 1>(acc[i], sm.col, sm.val, e, e + 1,
                                                                        xl, p.K, vm);
                            }
                        }
                    }
                }
                cur_blk = sm.next_blk;
                cur_k = sm.next_k;
                __syncthreads();
            }
            // ---- remainder row, tail entries, store ----
#pragma unroll
            for (int i = 0; i < RPG; ++i) {
                const int q = g + i * NG;
                if (q < R) {
                    const int32_t row = p.row_ids[rbase + r0 + q];
                    if (!p.skip_rem)
                        accumulate<S, VEC, VPT, LPR, U>(acc[i], p.rem_col, p.rem_val, p.rem_indptr[row],
                                                        p.rem_indptr[row + 1], xl, p.K, vm);
                    if (p.tail_nnz) {
                        const int64_t t0 = lower_bound_i32(p.tail_row, p.tail_nnz, row);
                        const int64_t t1 = lower_bound_i32(p.tail_row, p.tail_nnz, (int64_t)row + 1);
                        accumulate<S, VEC, VPT, LPR, 1>(acc[i], p.tail_col, p.tail_val, t0, t1, xl,
                                                        p.K, vm);
                    }
                    S *yr = yb + (int64_t)row * p.K + f0;
#pragma unroll
                    for (int v = 0; v < VPT; ++v)
                        if (vm[v]) {
                            if (p.skip_rem) {   // Y holds the row's remainder sum
                                const Frag<S, VEC> y0 = ldg_frag<S, VEC>(yr + v * LPR * VEC);
#pragma unroll
                                for (int q = 0; q < VEC; ++q) acc[i][v].v[q] = y0.v[q] + acc[i][v].v[q];
                            }
                            st_frag<S, VEC>(yr + v * LPR * VEC, acc[i][v]);
                        }
                }
            }
        }
    }
    }
}

// One CTA per row group; in add mode (skip_rem: most groups have nothing to
// add) each CTA walks a run of groups, so the empty ones cost one load each.
template <typename S, int VEC, int VPT, int LPR>
int launch_boo_n(BooParams<S> p, int64_t rg_first, int64_t rg_end, cudaStream_t s) {
    constexpr int SLAB = LPR * VPT * VEC;
    const int64_t slabs = ceil_div(p.K, SLAB);
    const int64_t n_rg = rg_end - rg_first;
    if (slabs > 65535 || n_rg > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    if (n_rg <= 0) return SPMM_OK;
    p.n_rg = rg_end;
    p.rg_first = rg_first;
    p.rgs_per_cta = 1;
    if (p.skip_rem) {
        int dev = 0, sms = 0;
        SPMM_CUDA_TRY(cudaGetDevice(&dev));
        SPMM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        p.rgs_per_cta = ceil_div(n_rg, (int64_t)sms * 8);
    }
    const int64_t ctas = ceil_div(n_rg, p.rgs_per_cta);
    dim3 grid((unsigned)ctas, (unsigned)slabs, (unsigned)(p.batch < 65535 ? p.batch : 65535));
    boo_spmm_kernel<S, VEC, VPT, LPR><<<grid, kBooThreads, 0, s>>>(p);
    SPMM_PRODUCT_LAUNCHED();
    return SPMM_OK;
}

// ---- load-balanced CSR remainder ------------------------------------------
//
// For matrices whose nonzeros are mostly in the CSR remainder (power-law
// graphs, uniform random; the reference's remainder kernel,
// boo_kernel.cu:905-937, runs one thread block per row) rows are skewed: up to
// tens of thousands of entries next to a median of ~20.  Three launches on the
// stream, each Y element written once and then updated once at most:
//   * the rows of at most kLongRow entries (rem_tile_kernel): warp tiles of 32
//       consecutive rows dealt round-robin to all warps; the tile's row
//       pointers in one coalesced load; per row the (column, value) pairs are
//       fetched 32 at a time by the lanes (the next row's first chunk while the
//       current row's X rows are in flight) and broadcast by shuffles, 8 / VPT
//       X rows in flight per warp;
//     it stores Y for every such row (zeros for empty rows);
//   * rem_long_kernel: a CTA per tile of 512 rows takes every longer row of
//     its tile; its 16 warps each sum a contiguous sixteenth of the row and the
//     CTA adds the partials in warp order and stores Y;
//   * the block kernel then adds blocks and tail entries into the row groups
//     that have any (skip_rem).
// Every result is deterministic.
constexpr int kLongRow = 1024;
constexpr int kRemWarps = 8;    // warps per CTA of the tile kernel
constexpr int kLongWarps = 16;  // warps sharing one long row, 16 / VPT X rows in flight each

// acc += sum over entries [e0, e1) of val * X[col]; (c, v) = this lane's
// entry e0 + lane (already loaded by the caller).
template <typename S, int VEC, int VPT, int U>
__device__ __forceinline__ void rem_span(Frag<S, VEC> (&acc)[VPT], const int32_t *col, const S *val, int64_t e0,
                                         int64_t e1, int32_t c, S v, const S *xl, int64_t K,
                                         const bool (&vm)[VPT], int lane) {
    constexpr int STR = 32 * VEC;   // U: X rows in flight per warp
    for (int64_t b = e0; b < e1; b += 32) {
        if (b != e0) {
            const int64_t e = b + lane;
            c = e < e1 ? __ldg(col + e) : 0;
            v = e < e1 ? __ldg(val + e) : S(0);
        }
        const int n = e1 - b < 32 ? (int)(e1 - b) : 32;
        // batches of U entries, the last one partial: its X rows are in flight
        // together too (a 5-entry row issues its five loads at once)
        for (int j = 0; j < n; j += U) {
            Frag<S, VEC> x[U][VPT];
            S a[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int32_t cu = __shfl_sync(kFullMask, c, (j + u) & 31);
                a[u] = __shfl_sync(kFullMask, v, (j + u) & 31);
                if (j + u < n) {   // warp-uniform
                    const S *xr = xl + (int64_t)cu * K;
#pragma unroll
                    for (int q = 0; q < VPT; ++q)
                        if (vm[q]) x[u][q] = ldg_frag<S, VEC>(xr + q * STR);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (j + u < n)
#pragma unroll
                    for (int q = 0; q < VPT; ++q)
                        if (vm[q])
#pragma unroll
                            for (int t = 0; t < VEC; ++t) acc[q].v[t] = fma(a[u], x[u][q].v[t], acc[q].v[t]);
        }
    }
}

template <typename S, int VEC, int VPT>
__device__ __forceinline__ void rem_store_row(S *yr, const Frag<S, VEC> (&acc)[VPT], const bool (&vm)[VPT]) {
    constexpr int STR = 32 * VEC;
#pragma unroll
    for (int q = 0; q < VPT; ++q)
        if (vm[q]) st_frag<S, VEC>(yr + q * STR, acc[q]);
}

template <typename S, int VEC, int VPT>
__global__ void __launch_bounds__(32 * kRemWarps, 2) rem_tile_kernel(const BooParams<S> p) {
    constexpr int SLAB = 32 * VPT * VEC;
    const int lane = threadIdx.x & 31;
    const int64_t f0 = (int64_t)blockIdx.y * SLAB + (int64_t)lane * VEC;
    bool vm[VPT];
#pragma unroll
    for (int q = 0; q < VPT; ++q) vm[q] = f0 + (int64_t)q * 32 * VEC < p.K;
    const int64_t nwarps = (int64_t)gridDim.x * kRemWarps;
    const int64_t ntiles = (p.rows + 31) / 32;
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K + f0;
        for (int64_t t = (int64_t)blockIdx.x * kRemWarps + (threadIdx.x >> 5); t < ntiles; t += nwarps) {
            const int64_t r0 = t * 32;
            const int nrow = p.rows - r0 < 32 ? (int)(p.rows - r0) : 32;
            // row pointers of the tile: lane l holds rows r0 + l's [e0, e1)
            const int64_t me0 = lane < nrow ? (int64_t)__ldg(p.rem_indptr + r0 + lane) : 0;
            const int64_t me1 = lane < nrow ? (int64_t)__ldg(p.rem_indptr + r0 + lane + 1) : 0;
            // first chunk of the first row
            int64_t e0 = __shfl_sync(kFullMask, me0, 0), e1 = __shfl_sync(kFullMask, me1, 0);
            int32_t c = e0 + lane < e1 ? __ldg(p.rem_col + e0 + lane) : 0;
            S v = e0 + lane < e1 ? __ldg(p.rem_val + e0 + lane) : S(0);
            for (int j = 0; j < nrow; ++j) {
                // the next row's first chunk, loaded while this row runs
                int64_t n0 = 0, n1 = 0;
                int32_t nc = 0;
                S nv = S(0);
                if (j + 1 < nrow) {
                    n0 = __shfl_sync(kFullMask, me0, j + 1);
                    n1 = __shfl_sync(kFullMask, me1, j + 1);
                    if (n1 - n0 <= kLongRow && n0 + lane < n1) {
                        nc = __ldg(p.rem_col + n0 + lane);
                        nv = __ldg(p.rem_val + n0 + lane);
                    }
                }
                if (e1 - e0 <= kLongRow) {   // longer rows: rem_long_kernel
                    Frag<S, VEC> acc[VPT];
#pragma unroll
                    for (int q = 0; q < VPT; ++q)
#pragma unroll
                        for (int u = 0; u < VEC; ++u) acc[q].v[u] = S(0);
                    rem_span<S, VEC, VPT, 8 / VPT>(acc, p.rem_col, p.rem_val, e0, e1, c, v, xl, p.K, vm, lane);
                    rem_store_row<S, VEC, VPT>(yb + (r0 + j) * p.K, acc, vm);
                }
                e0 = n0;
                e1 = n1;
                c = nc;
                v = nv;
            }
        }
    }
}


// ---- short rows through the plan's row view ----
//
// Matrices of a few entries per row (a 2-D Laplacian: 5) are latency bound in
// the block kernel: a CTA walks its group's blocks through shared memory in a
// chain of dependent loads.  With the plan's row-ordered copy of every entry
// a warp takes one row: its row pointers, its (column, value) pairs in one
// coalesced load, then every X row of the row in flight at once.  Warps take
// the positions of row groups [rg0, rg1) in the row-group order (row =
// row_ids[k]), so a range covers exactly its rows.  float32 with one vector
// per lane: 24 warps per SM, X rows in batches of 6 to stay within the
// registers (2-D Laplacian 0.051 -> 0.041 ms against 16 warps per SM with
// batches of 8); other shapes keep 16 warps per SM and batches of 8.
constexpr int kShortWarps = 8;

// Blocks per SM of row_warp_kernel: float32 rows of one vector per lane fit
// three (X rows in batches of 6); other shapes two (batches of 8).
template <typename S, int VPT>
__host__ __device__ constexpr int row_warp_ctas() { return VPT == 1 && sizeof(S) == 4 ? 3 : 2; }

template <typename S, int VEC, int VPT>
__global__ void __launch_bounds__(32 * kShortWarps, row_warp_ctas<S, VPT>()) row_warp_kernel(const BooParams<S> p, int64_t rg0, int64_t rg1, const int32_t *__restrict__ ident) {
    constexpr int SLAB = 32 * VPT * VEC;
    const int lane = threadIdx.x & 31;
    const int64_t f0 = (int64_t)blockIdx.y * SLAB + (int64_t)lane * VEC;
    bool vm[VPT];
#pragma unroll
    for (int q = 0; q < VPT; ++q) vm[q] = f0 + (int64_t)q * 32 * VEC < p.K;
    const int64_t nwarps = (int64_t)gridDim.x * kShortWarps;
    const int64_t k0 = __ldg(p.row_grp_ptr + rg0), k1 = __ldg(p.row_grp_ptr + rg1);
    const bool same = __ldg(ident) != 0;   // row_ids[k] == k: one dependent load less per row
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K + f0;
        int64_t k = k0 + (int64_t)blockIdx.x * kShortWarps + (threadIdx.x >> 5);
        // Software pipeline over this warp's rows k, k + nwarps, ...: while a
        // row's X rows are in flight, the next row's (column, value) pairs and
        // the range of the row after it are fetched, so a row costs one load
        // latency, not three.
        int64_t row = 0, e0 = 0, e1 = 0;
        int32_t c = 0;
        S v = S(0);
        if (k < k1) {
            row = same ? k : (int64_t)__ldg(p.row_ids + k);
            e0 = __ldg(p.rem_indptr + row);
            e1 = __ldg(p.rem_indptr + row + 1);
            c = e0 + lane < e1 ? __ldg(p.rem_col + e0 + lane) : 0;
            v = e0 + lane < e1 ? __ldg(p.rem_val + e0 + lane) : S(0);
        }
        int64_t nrow = 0, n0 = 0, n1 = 0;
        if (k + nwarps < k1) {
            nrow = same ? k + nwarps : (int64_t)__ldg(p.row_ids + k + nwarps);
            n0 = __ldg(p.rem_indptr + nrow);
            n1 = __ldg(p.rem_indptr + nrow + 1);
        }
        for (; k < k1; k += nwarps) {
            int32_t nc = 0;
            S nv = S(0);
            if (k + nwarps < k1 && n0 + lane < n1) {
                nc = __ldg(p.rem_col + n0 + lane);
                nv = __ldg(p.rem_val + n0 + lane);
            }
            int64_t mrow = 0, m0 = 0, m1 = 0;
            if (k + 2 * nwarps < k1) {
                mrow = same ? k + 2 * nwarps : (int64_t)__ldg(p.row_ids + k + 2 * nwarps);
                m0 = __ldg(p.rem_indptr + mrow);
                m1 = __ldg(p.rem_indptr + mrow + 1);
            }
            Frag<S, VEC> acc[VPT];
#pragma unroll
            for (int q = 0; q < VPT; ++q)
#pragma unroll
                for (int u = 0; u < VEC; ++u) acc[q].v[u] = S(0);
            rem_span<S, VEC, VPT, row_warp_ctas<S, VPT>() == 3 ? 6 : 8 / VPT>(acc, p.rem_col, p.rem_val, e0, e1, c, v, xl, p.K, vm, lane);
            rem_store_row<S, VEC, VPT>(yb + row * p.K, acc, vm);
            row = nrow;
            e0 = n0;
            e1 = n1;
            c = nc;
            v = nv;
            nrow = mrow;
            n0 = m0;
            n1 = m1;
        }
    }
}

template <typename S, int VEC, int VPT>
int launch_row_warp(const BooParams<S> &p, int64_t rg0, int64_t rg1, int64_t max_nr, const int32_t *ident,
                    cudaStream_t s) {
    constexpr int SLAB = 32 * VPT * VEC;
    const int64_t slabs = ceil_div(p.K, SLAB);
    if (slabs > 65535) return SPMM_EUNSUPPORTED;
    if (rg1 <= rg0) return SPMM_OK;
    int dev = 0, sms = 0;
    SPMM_CUDA_TRY(cudaGetDevice(&dev));
    SPMM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t bound = (rg1 - rg0) * max_nr < p.rows ? (rg1 - rg0) * max_nr : p.rows;   // rows of the range
    const int64_t want = ceil_div(bound > 0 ? bound : 1, (int64_t)kShortWarps);
    const int64_t cap = (int64_t)sms * row_warp_ctas<S, VPT>();   // resident CTAs: warps walk their rows pipelined
    const unsigned bz = (unsigned)(p.batch < 65535 ? p.batch : 65535);
    dim3 grid((unsigned)(want < cap ? want : cap), (unsigned)slabs, bz);
    row_warp_kernel<S, VEC, VPT><<<grid, 32 * kShortWarps, 0, s>>>(p, rg0, rg1, ident);
    SPMM_PRODUCT_LAUNCHED();
    return SPMM_OK;
}

template <typename S>
int row_warp_dispatch(const BooParams<S> &p, int64_t rg0, int64_t rg1, int64_t max_nr, const int32_t *ident,
                      bool aligned, cudaStream_t s) {
    constexpr int V = 16 / (int)sizeof(S);
    if (aligned && p.K % V == 0) {
        if (p.K <= 32 * V) return launch_row_warp<S, V, 1>(p, rg0, rg1, max_nr, ident, s);
        return launch_row_warp<S, V, 2>(p, rg0, rg1, max_nr, ident, s);
    }
    return launch_row_warp<S, 1, 4>(p, rg0, rg1, max_nr, ident, s);
}

// Narrow features (K <= 16 VEC, e.g. 64 floats): half a warp per row, two
// rows per warp, so no lane idles.  Each half loads its row's (column, value)
// pairs 16 at a time and hands them out by 16-wide shuffles; the warp walks to
// the longer of its two rows (a uniform trip count keeps the shuffles
// converged), each half predicating its own entries, 8 X rows in flight.
// Rows of more than kLongRow entries are left to rem_long_kernel when
// skip_long is set.
template <typename S, int VEC>
__global__ void __launch_bounds__(256, 2) row_half_kernel(const BooParams<S> p, int skip_long) {
    constexpr int U = 8;
    const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
    const int64_t f0 = (int64_t)hl * VEC;
    const bool fm = f0 < p.K;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t npairs = (p.rows + 1) / 2;
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K + f0;
        for (int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); q < npairs; q += nwarps) {
            const int64_t k = 2 * q + half;
            const bool valid = k < p.rows;
            const int64_t row = valid ? (int64_t)__ldg(p.row_ids + k) : 0;
            const int64_t e0 = valid ? (int64_t)__ldg(p.rem_indptr + row) : 0;
            int64_t n = valid ? (int64_t)__ldg(p.rem_indptr + row + 1) - e0 : 0;
            const bool mine = valid && !(skip_long && n > kLongRow);
            if (!mine) n = 0;
            int64_t nmax = n;
            const int64_t other = __shfl_xor_sync(kFullMask, nmax, 16);
            nmax = other > nmax ? other : nmax;
            Frag<S, VEC> acc;
#pragma unroll
            for (int t = 0; t < VEC; ++t) acc.v[t] = S(0);
            for (int64_t b = 0; b < nmax; b += 16) {
                const int32_t c = b + hl < n ? __ldg(p.rem_col + e0 + b + hl) : 0;
                const S v = b + hl < n ? __ldg(p.rem_val + e0 + b + hl) : S(0);
                const int m = nmax - b < 16 ? (int)(nmax - b) : 16;                 // uniform
                const int mh = n - b < 16 ? (n - b > 0 ? (int)(n - b) : 0) : 16;     // this half's
                for (int j = 0; j < m; j += U) {
                    Frag<S, VEC> x[U];
                    S a[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int32_t cu = __shfl_sync(kFullMask, c, (j + u) & 15, 16);
                        a[u] = __shfl_sync(kFullMask, v, (j + u) & 15, 16);
                        if (j + u < mh && fm) x[u] = ldg_frag<S, VEC>(xl + (int64_t)cu * p.K);
                    }
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        if (j + u < mh && fm)
#pragma unroll
                            for (int t = 0; t < VEC; ++t) acc.v[t] = fma(a[u], x[u].v[t], acc.v[t]);
                }
            }
            if (mine && fm) st_frag<S, VEC>(yb + row * p.K, acc);
        }
    }
}

template <typename S, int VEC>
int launch_row_half(const BooParams<S> &p, int skip_long, cudaStream_t s) {
    if (p.rows <= 0) return SPMM_OK;
    int dev = 0, sms = 0;
    SPMM_CUDA_TRY(cudaGetDevice(&dev));
    SPMM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t want = ceil_div((p.rows + 1) / 2, (int64_t)8);
    const int64_t cap = (int64_t)sms * 2 * 4;   // a few waves of resident CTAs
    const unsigned bz = (unsigned)(p.batch < 65535 ? p.batch : 65535);
    row_half_kernel<S, VEC><<<dim3((unsigned)(want < cap ? want : cap), 1, bz), 256, 0, s>>>(p, skip_long);
    SPMM_PRODUCT_LAUNCHED();
    return SPMM_OK;
}

// ---- nnz-flat remainder (default on the aligned path) ----
//
// The CSR remainder is cut into chunks of `chunk` consecutive entries,
// whatever the rows (merge-path style), so every warp gets the same work
// whatever the row lengths (power-law rows of 3 to 20k entries):
//   * rem_flat_plan_kernel: the row holding each chunk's first entry, and
//     zeros for the rows without entries;
//   * rem_flat_kernel: warps take chunks round-robin and walk their entries
//     with the X rows landing in shared memory through asynchronous copies
//     (cp.async, 16 bytes per lane), so the X rows in flight are bounded by
//     shared memory (kAsyncBuf batches of kAsyncBatch rows per warp) rather
//     than by the register file: per batch the lanes read the (column, value)
//     pairs one batch ahead and every lane copies its features of each X row
//     slab as one commit group; the warp consumes the batches in order (each
//     lane reads back only the bytes it copied itself) and refills the freed
//     buffer.  A row lying inside the chunk is stored to Y; a row cut by the
//     chunk's start goes to the chunk's partial row 0, a row cut only by its
//     end to partial row 1;
//   * rem_flat_fix_kernel: each row cut by chunk boundaries gets the sum of
//     its partials in chunk order.
// Sums run in entry order within a chunk; the result is deterministic.
constexpr int kAsyncBatch = 4;   // X rows per batch (one commit group)
constexpr int kAsyncBuf = 2;     // batches in flight per warp

template <typename S, int VEC, int VPT>
struct AsyncShape {
    static constexpr int kSlab = 32 * VPT * VEC;                      // features per launch slice
    static constexpr int kSlotBytes = kSlab * (int)sizeof(S);
    static constexpr int kWarpBytes = kAsyncBuf * kAsyncBatch * kSlotBytes;
    static constexpr int kWarps = (192 * 1024) / kWarpBytes < 24 ? (192 * 1024) / kWarpBytes : 24;
    static constexpr int kThreads = 32 * kWarps;
    // per warp, after every warp's slots: entry rows | entry values
    static constexpr int kValsOff = kAsyncBuf * kAsyncBatch * 4;
    static constexpr int kMetaBytes = (kValsOff + kAsyncBuf * kAsyncBatch * (int)sizeof(S) + 15) / 16 * 16;
    static constexpr int kSmem = kWarps * (kWarpBytes + kMetaBytes) + 128;
    static_assert(kWarps >= 4, "flat remainder: at least four warps per CTA");
    static_assert(kWarpBytes % 128 == 0 && kValsOff % 8 == 0, "flat remainder: smem alignment");
};

// Warp per 32 rows: zeros for the empty rows (every batch), and chunk_row[c]
// = r for every chunk c whose first entry c * chunk lies in row r.
template <typename S, int VEC>
__global__ void __launch_bounds__(256) rem_flat_plan_kernel(const BooParams<S> p) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * 8;
    const int64_t ntiles = (p.rows + 31) / 32;
    for (int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); t < ntiles; t += nwarps) {
        const int64_t r = t * 32 + lane;
        int32_t e0 = 0, e1 = 0;
        if (r < p.rows) {
            e0 = __ldg(p.rem_indptr + r);
            e1 = __ldg(p.rem_indptr + r + 1);
        }
        if (e1 > e0)
            for (int64_t c = (e0 + (int64_t)p.chunk - 1) / p.chunk; c * p.chunk < e1; ++c)
                p.chunk_row[c] = (int32_t)r;
        unsigned em = __ballot_sync(kFullMask, r < p.rows && e0 == e1);
        while (em) {
            const int l = __ffs(em) - 1;
            em &= em - 1;
            const int64_t row = t * 32 + l;
            for (int64_t bt = 0; bt < p.batch; ++bt) {
                S *yr = p.Y + (bt * p.rows + row) * p.K;
                for (int64_t f = (int64_t)lane * VEC; f < p.K; f += 32 * VEC) {
                    Frag<S, VEC> z;
#pragma unroll
                    for (int u = 0; u < VEC; ++u) z.v[u] = S(0);
                    st_frag<S, VEC>(yr + f, z);
                }
            }
        }
    }
}

template <typename S, int VEC, int VPT>
__global__ void __launch_bounds__(AsyncShape<S, VEC, VPT>::kThreads, 1) rem_flat_kernel(const BooParams<S> p) {
    using Sh = AsyncShape<S, VEC, VPT>;
    constexpr int STR = 32 * VEC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 127) & ~(uintptr_t)127);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    S *slots = reinterpret_cast<S *>(base + warp * Sh::kWarpBytes);
    uint8_t *meta = base + Sh::kWarps * Sh::kWarpBytes + warp * Sh::kMetaBytes;
    int32_t *erow = reinterpret_cast<int32_t *>(meta);   // row per slot, -1: none
    S *eval = reinterpret_cast<S *>(meta + Sh::kValsOff);

    const int64_t f0 = (int64_t)blockIdx.y * Sh::kSlab + (int64_t)lane * VEC;
    bool vm[VPT];
#pragma unroll
    for (int q = 0; q < VPT; ++q) vm[q] = f0 + (int64_t)q * STR < p.K;
    const int64_t nwarps = (int64_t)gridDim.x * Sh::kWarps;
    uint32_t nb = 0;   // batches this warp has issued (every chunk): buffer = nb % kAsyncBuf
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K + f0;
        for (int64_t c = (int64_t)blockIdx.x * Sh::kWarps + warp; c < p.nch; c += nwarps) {
            const int32_t E0 = (int32_t)(c * p.chunk);
            const int32_t E1 = (int32_t)(p.rem_nnz - (int64_t)E0 < p.chunk ? p.rem_nnz : (int64_t)E0 + p.chunk);
            const int32_t rs = p.chunk_row[c];
            // window of 32 rows from wb: lane l holds row wb + l's entries [me0, me1)
            int64_t wb = rs;
            int32_t me0 = INT_MAX, me1 = INT_MAX;
            auto load_window = [&]() {
                me0 = me1 = INT_MAX;
                if (wb + lane < p.rows) {
                    me0 = __ldg(p.rem_indptr + wb + lane);
                    me1 = __ldg(p.rem_indptr + wb + lane + 1);
                }
            };
            load_window();
            const bool rs_cut = __shfl_sync(kFullMask, me0, 0) < E0;   // row rs began in an earlier chunk
            int32_t pos = E0;   // stream position of the prepared batch
            // the prepared batch: pn entries, lane j < pn holds entry pos + j
            int prow = -1, pn = 0;
            int32_t pc = 0;
            S pv = S(0);
            auto prepare = [&]() {
                prow = -1;
                pn = 0;
                pc = 0;
                pv = S(0);
                if (pos >= E1) return;
                int32_t wend = __shfl_sync(kFullMask, me1, 31);
                while (pos >= wend) {   // the window's rows all end at or before pos
                    wb += 32;
                    load_window();
                    wend = __shfl_sync(kFullMask, me1, 31);
                }
                const int32_t lim = E1 < wend ? E1 : wend;
                pn = lim - pos < kAsyncBatch ? lim - pos : kAsyncBatch;
                int r = 0;
#pragma unroll
                for (int j = 0; j < kAsyncBatch; ++j) {
                    const int rj = __popc(__ballot_sync(kFullMask, me1 <= pos + j));   // rows ending before
                    if (lane == j) r = rj;
                }
                if (lane < pn) {
                    prow = (int)(wb + r);
                    pc = __ldg(p.rem_col + pos + lane);
                    pv = __ldg(p.rem_val + pos + lane);
                }
            };
            // Copies the prepared batch into buffer b and commits one group
            // (empty once the chunk is done); false when it was empty.
            auto issue = [&](uint32_t b) -> bool {
                if (pn == 0) {
                    cp_async_commit();
                    return false;
                }
                __syncwarp();   // the previous readers of this buffer's metadata are done
                if (lane < kAsyncBatch) {
                    erow[b * kAsyncBatch + lane] = prow;
                    eval[b * kAsyncBatch + lane] = pv;
                }
                S *dst = slots + (size_t)(b * kAsyncBatch) * Sh::kSlab + lane * VEC;
#pragma unroll
                for (int j = 0; j < kAsyncBatch; ++j) {
                    const int32_t cj = __shfl_sync(kFullMask, pc, j);
                    if (j < pn) {
                        const S *src = xl + (int64_t)cj * p.K;
#pragma unroll
                        for (int qq = 0; qq < VPT; ++qq)
                            if (vm[qq]) cp_async16(dst + j * Sh::kSlab + qq * STR, src + qq * STR);
                    }
                }
                cp_async_commit();
                pos += pn;
                prepare();
                return true;
            };
            prepare();
            uint32_t issued = 0;   // non-empty batches of this chunk
            bool more = true;
            for (int i = 0; i < kAsyncBuf; ++i) {   // prologue: kAsyncBuf groups
                if (more && issue((nb + issued) % kAsyncBuf)) ++issued;
                else if (more) more = false;
                else cp_async_commit();
            }
            Frag<S, VEC> acc[VPT];
#pragma unroll
            for (int q = 0; q < VPT; ++q)
#pragma unroll
                for (int u = 0; u < VEC; ++u) acc[q].v[u] = S(0);
            int cur = -1;
            // a finished row: to Y, or to a partial row when a chunk boundary cuts it
            S *pb = p.part + ((bt * p.nch + c) * 2) * p.K + f0;
            auto flush = [&](bool last_cut) {
                S *dst = yb + (int64_t)cur * p.K;
                if (cur == rs && rs_cut) dst = pb;
                else if (last_cut) dst = pb + p.K;
                rem_store_row<S, VEC, VPT>(dst, acc, vm);
            };
            for (uint32_t k = 0; k < issued; ++k) {
                const uint32_t b = (nb + k) % kAsyncBuf;
                cp_async_wait<kAsyncBuf - 1>();   // batch k's group (every later one may pend)
                __syncwarp();
                const S *slot = slots + (size_t)(b * kAsyncBatch) * Sh::kSlab + lane * VEC;
#pragma unroll
                for (int j = 0; j < kAsyncBatch; ++j) {
                    const int r = erow[b * kAsyncBatch + j];
                    if (r < 0) break;
                    if (r != cur) {
                        if (cur >= 0) flush(false);
#pragma unroll
                        for (int q = 0; q < VPT; ++q)
#pragma unroll
                            for (int u = 0; u < VEC; ++u) acc[q].v[u] = S(0);
                        cur = r;
                    }
                    const S a = eval[b * kAsyncBatch + j];
#pragma unroll
                    for (int q = 0; q < VPT; ++q)
                        if (vm[q]) {
                            const Frag<S, VEC> x = lds_frag<S, VEC>(slot + j * Sh::kSlab + q * STR);
#pragma unroll
                            for (int u = 0; u < VEC; ++u) acc[q].v[u] = fma(a, x.v[u], acc[q].v[u]);
                        }
                }
                // refill this buffer (one group, empty once the chunk is done)
                if (more) {
                    if (issue(b)) ++issued;
                    else more = false;
                } else {
                    cp_async_commit();
                }
            }
            if (cur >= 0) flush(__ldg(p.rem_indptr + cur + 1) > E1);
            nb += issued;
        }
    }
    cp_async_wait<0>();
}

// Warp per chunk c >= 1 whose first row r began in chunk c - 1: Y[r] = its
// partial there (row 1: cut by that chunk's end) plus its partial rows 0 of
// chunks c, c + 1, ... while r holds their first entry.
template <typename S, int VEC>
__global__ void __launch_bounds__(256) rem_flat_fix_kernel(const BooParams<S> p) {
    const int lane = threadIdx.x & 31;
    const int64_t nwarps = (int64_t)gridDim.x * 8;
    for (int64_t c = 1 + (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); c < p.nch; c += nwarps) {
        const int32_t r = p.chunk_row[c];
        const int64_t s0 = __ldg(p.rem_indptr + r), e0c = c * (int64_t)p.chunk;
        if (s0 >= e0c || s0 < e0c - p.chunk) continue;   // not cut here, or cut first at an earlier boundary
        int64_t c1 = c;
        while (c1 + 1 < p.nch && p.chunk_row[c1 + 1] == r) ++c1;
        for (int64_t bt = 0; bt < p.batch; ++bt) {
            const S *pp = p.part + (bt * p.nch) * 2 * p.K;
            S *yr = p.Y + (bt * p.rows + r) * p.K;
            for (int64_t f = (int64_t)lane * VEC; f < p.K; f += 32 * VEC) {
                Frag<S, VEC> acc = ldg_frag<S, VEC>(pp + ((c - 1) * 2 + 1) * p.K + f);
                for (int64_t cc = c; cc <= c1; ++cc) {
                    const Frag<S, VEC> t = ldg_frag<S, VEC>(pp + (cc * 2) * p.K + f);
#pragma unroll
                    for (int u = 0; u < VEC; ++u) acc.v[u] += t.v[u];
                }
                st_frag<S, VEC>(yr + f, acc);
            }
        }
    }
}

template <typename S, int VEC, int VPT>
__global__ void __launch_bounds__(32 * kLongWarps, 1) rem_long_kernel(const BooParams<S> p) {
    constexpr int SLAB = 32 * VPT * VEC;
    __shared__ Frag<S, VEC> part[kLongWarps][VPT][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t f0 = (int64_t)blockIdx.y * SLAB + (int64_t)lane * VEC;
    bool vm[VPT];
#pragma unroll
    for (int q = 0; q < VPT; ++q) vm[q] = f0 + (int64_t)q * 32 * VEC < p.K;
    const int64_t r0 = (int64_t)blockIdx.x * 32 * kLongWarps;
    const int64_t myrow = r0 + threadIdx.x;
    const bool is_long = myrow < p.rows &&
                         __ldg(p.rem_indptr + myrow + 1) - __ldg(p.rem_indptr + myrow) > kLongRow;
    if (!__syncthreads_or(is_long)) return;
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K + f0;
        for (int64_t row = r0; row < r0 + 32 * kLongWarps && row < p.rows; ++row) {
            const int64_t e0 = __ldg(p.rem_indptr + row), e1 = __ldg(p.rem_indptr + row + 1);
            if (e1 - e0 <= kLongRow) continue;
            // warp w: entries [e0 + w*len/W, e0 + (w+1)*len/W)
            const int64_t len = e1 - e0;
            const int64_t a = e0 + len * warp / kLongWarps, b = e0 + len * (warp + 1) / kLongWarps;
            Frag<S, VEC> acc[VPT];
#pragma unroll
            for (int q = 0; q < VPT; ++q)
#pragma unroll
                for (int t = 0; t < VEC; ++t) acc[q].v[t] = S(0);
            const int32_t c = a + lane < b ? __ldg(p.rem_col + a + lane) : 0;
            const S v = a + lane < b ? __ldg(p.rem_val + a + lane) : S(0);
            rem_span<S, VEC, VPT, 16 / VPT>(acc, p.rem_col, p.rem_val, a, b, c, v, xl, p.K, vm, lane);
#pragma unroll
            for (int q = 0; q < VPT; ++q) part[warp][q][lane] = acc[q];
            __syncthreads();
            if (warp == 0) {
#pragma unroll
                for (int q = 0; q < VPT; ++q) {
                    Frag<S, VEC> t = part[0][q][lane];
#pragma unroll
                    for (int w = 1; w < kLongWarps; ++w)
#pragma unroll
                        for (int u = 0; u < VEC; ++u) t.v[u] += part[w][q][lane].v[u];
                    acc[q] = t;
                }
                rem_store_row<S, VEC, VPT>(yb + row * p.K, acc, vm);
            }
            __syncthreads();
        }
    }
}

// Chunk size of the nnz-flat remainder: about 8192 chunks, 256..2048 entries.
inline int32_t rem_flat_chunk(int64_t rem_nnz) {
    const int64_t c = ceil_div(rem_nnz, (int64_t)8192);
    return (int32_t)(c < 256 ? 256 : c > 2048 ? 2048 : c);
}

// Scratch of the nnz-flat remainder: chunk rows, then two partial rows of K
// per (batch, chunk).
inline size_t rem_flat_workspace(int64_t rem_nnz, int64_t batch, int64_t K, size_t elem) {
    if (rem_nnz <= 0) return 0;
    const int64_t nch = ceil_div(rem_nnz, (int64_t)rem_flat_chunk(rem_nnz));
    return (size_t)ceil_div(nch * 4, (int64_t)256) * 256 + (size_t)(batch * nch * 2 * K) * elem;
}

// The nnz-flat remainder (plan, chunks, fix-up) on the caller's scratch `ws`
// (rem_flat_workspace() bytes, checked by the caller).
template <typename S, int VEC, int VPT>
int launch_rem_flat(BooParams<S> p, int sms, unsigned bz, void *ws, cudaStream_t s) {
    using Sh = AsyncShape<S, VEC, VPT>;
    const int64_t slabs = ceil_div(p.K, (int64_t)Sh::kSlab);
    if (slabs > 65535 || p.rem_nnz > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    p.chunk = rem_flat_chunk(p.rem_nnz);
    p.nch = ceil_div(p.rem_nnz, (int64_t)p.chunk);
    p.chunk_row = reinterpret_cast<int32_t *>(ws);
    p.part = reinterpret_cast<S *>(reinterpret_cast<uint8_t *>(ws) + ceil_div(p.nch * 4, (int64_t)256) * 256);
    auto kern = rem_flat_kernel<S, VEC, VPT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Sh::kSmem);
    const int64_t tiles = ceil_div(p.rows, (int64_t)32);
    const int64_t gp = ceil_div(tiles, (int64_t)8) < (int64_t)sms * 8 ? ceil_div(tiles, (int64_t)8) : (int64_t)sms * 8;
    if (e == cudaSuccess) {
        rem_flat_plan_kernel<S, VEC><<<(unsigned)gp, 256, 0, s>>>(p);
        e = cudaGetLastError();
        if (e == cudaSuccess) note_product_launch();
    }
    if (e == cudaSuccess) {
        const int64_t ctas = ceil_div(p.nch, (int64_t)Sh::kWarps);
        const int64_t g = ctas < (int64_t)sms ? ctas : (int64_t)sms;
        kern<<<dim3((unsigned)g, (unsigned)slabs, bz), Sh::kThreads, Sh::kSmem, s>>>(p);
        e = cudaGetLastError();
        if (e == cudaSuccess) note_product_launch();
    }
    if (e == cudaSuccess) {
        const int64_t gf = ceil_div(p.nch, (int64_t)8) < (int64_t)sms * 8 ? ceil_div(p.nch, (int64_t)8) : (int64_t)sms * 8;
        rem_flat_fix_kernel<S, VEC><<<(unsigned)(gf > 0 ? gf : 1), 256, 0, s>>>(p);
        e = cudaGetLastError();
        if (e == cudaSuccess) note_product_launch();
    }
    return e == cudaSuccess ? SPMM_OK : SPMM_ECUDA;
}

// The CSR remainder of every row into Y: nnz-flat chunks (`flat`: aligned X
// and Y, the default), else rows of at most kLongRow entries at full width
// through registers, then the long rows.
template <typename S, int VEC, int VPT>
int launch_rem(const BooParams<S> &p, bool flat, bool by_row, void *ws, cudaStream_t s) {
    constexpr int SLAB = 32 * VPT * VEC;
    const int64_t slabs = ceil_div(p.K, SLAB);
    if (slabs > 65535) return SPMM_EUNSUPPORTED;
    int dev = 0, sms = 0;
    SPMM_CUDA_TRY(cudaGetDevice(&dev));
    SPMM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const unsigned bz = (unsigned)(p.batch < 65535 ? p.batch : 65535);
    if constexpr (VEC > 1) {
        if (flat) return launch_rem_flat<S, VEC, VPT>(p, sms, bz, ws, s);
    }
    if constexpr (VEC > 1) {
        if (by_row) {   // narrow features, short rows: half a warp per row; long rows below
            const int rc = launch_row_half<S, VEC>(p, 1, s);
            if (rc != SPMM_OK) return rc;
        }
    }
    if (!by_row || VEC == 1) {
        const int64_t tile_ctas = ceil_div(ceil_div(p.rows, (int64_t)32), (int64_t)kRemWarps);
        const int64_t g1 = tile_ctas < (int64_t)sms * 8 ? tile_ctas : (int64_t)sms * 8;
        rem_tile_kernel<S, VEC, VPT><<<dim3((unsigned)g1, (unsigned)slabs, bz), 32 * kRemWarps, 0, s>>>(p);
        SPMM_PRODUCT_LAUNCHED();
    }
    const int64_t g2 = ceil_div(p.rows, (int64_t)(32 * kLongWarps));
    if (g2 > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    rem_long_kernel<S, VEC, VPT><<<dim3((unsigned)g2, (unsigned)slabs, bz), 32 * kLongWarps, 0, s>>>(p);
    SPMM_PRODUCT_LAUNCHED();
    return SPMM_OK;
}

// Vector width of the remainder pass: 16-byte X / Y accesses when both are
// 16-byte aligned and K is a multiple of the vector; 1 otherwise.
template <typename S>
constexpr int rem_vec() { return 16 / (int)sizeof(S); }

// Remainders of at most kShortRow entries per row on average with narrow
// features (K <= 16 vectors: one half warp covers a row) go half a warp per
// row by default; slab_features > 0 forces the nnz-flat chunks, < 0 the
// register path.
template <typename S>
bool rem_by_row(const BooParams<S> &p, bool aligned, int slab_req) {
    return aligned && slab_req == 0 && p.K % rem_vec<S>() == 0 && p.K <= 16 * rem_vec<S>() &&
           p.rem_nnz <= kShortRow * p.rows;
}

template <typename S>
bool rem_flat_applies(const BooParams<S> &p, bool aligned, int slab_req) {
    return aligned && p.K % rem_vec<S>() == 0 && slab_req >= 0 && !rem_by_row(p, aligned, slab_req);
}

template <typename S>
int rem_dispatch(const BooParams<S> &p, bool aligned, int slab_req, void *ws, cudaStream_t s) {
    constexpr int V = rem_vec<S>();
    const bool flat = rem_flat_applies(p, aligned, slab_req);
    const bool by_row = rem_by_row(p, aligned, slab_req);
    if (aligned && p.K % V == 0) {
        if (p.K <= 32 * V) return launch_rem<S, V, 1>(p, flat, by_row, ws, s);
        return launch_rem<S, V, 2>(p, flat, by_row, ws, s);
    }
    return launch_rem<S, 1, 4>(p, false, false, ws, s);
}

template <typename S>
int boo_dispatch(const BooParams<S> &p, int64_t rg0, int64_t rg1, bool aligned, cudaStream_t s);

template <>
int boo_dispatch<float>(const BooParams<float> &p, int64_t rg0, int64_t rg1, bool aligned, cudaStream_t s) {
    const int64_t K = p.K;
    if (aligned && K % 4 == 0) {
        if (K <= 32) return launch_boo_n<float, 4, 1, 8>(p, rg0, rg1, s);
        if (K <= 64) return launch_boo_n<float, 4, 1, 16>(p, rg0, rg1, s);
        if (K <= 128) return launch_boo_n<float, 4, 1, 32>(p, rg0, rg1, s);
        if (K <= 256) return launch_boo_n<float, 4, 2, 32>(p, rg0, rg1, s);
        return launch_boo_n<float, 4, 4, 32>(p, rg0, rg1, s);
    }
    if (K <= 32) return launch_boo_n<float, 1, 1, 32>(p, rg0, rg1, s);
    if (K <= 64) return launch_boo_n<float, 1, 2, 32>(p, rg0, rg1, s);
    return launch_boo_n<float, 1, 4, 32>(p, rg0, rg1, s);
}

template <>
int boo_dispatch<double>(const BooParams<double> &p, int64_t rg0, int64_t rg1, bool aligned, cudaStream_t s) {
    const int64_t K = p.K;
    if (aligned && K % 2 == 0) {
        if (K <= 16) return launch_boo_n<double, 2, 1, 8>(p, rg0, rg1, s);
        if (K <= 32) return launch_boo_n<double, 2, 1, 16>(p, rg0, rg1, s);
        if (K <= 64) return launch_boo_n<double, 2, 1, 32>(p, rg0, rg1, s);
        if (K <= 128) return launch_boo_n<double, 2, 2, 32>(p, rg0, rg1, s);
        return launch_boo_n<double, 2, 4, 32>(p, rg0, rg1, s);
    }
    if (K <= 32) return launch_boo_n<double, 1, 1, 32>(p, rg0, rg1, s);
    if (K <= 64) return launch_boo_n<double, 1, 2, 32>(p, rg0, rg1, s);
    return launch_boo_n<double, 1, 4, 32>(p, rg0, rg1, s);
}

// AUTO: the tensor-core kernel wins (measured on B200) when blocks (up to
// 64 x 64) hold on average >= 96 nonzeros: FEM 786k rows 1.83 vs 4.28 ms, 4096
// dense 64 x 64 blocks at K = 512 1.82 vs 3.12 ms; a 2-D Laplacian (~53 per
// block) stays on CUDA cores (0.105 vs 0.130 ms).
bool tc_selected(const spmm_boo_dev *A, int engine) {
    if (A->scalar_type != SPMM_F32 || engine == SPMM_ENGINE_CUDA_CORES) return false;
    if (engine >= SPMM_ENGINE_TENSOR_CORES) return true;
    return A->max_nr <= 64 && A->max_nc <= 64 && A->nb > 0 && A->nnz_c >= 96 * A->nb;
}

template <typename S>
int boo_matmul_impl(const spmm_boo_dev *A, const void *X, void *Y, int64_t batch, int64_t K, int64_t rg0,
                    int64_t rg1, int engine, const spmm_launch_cfg *cfg, cudaStream_t s) {
    void *ws = cfg ? cfg->workspace : nullptr;
    const size_t ws_bytes = cfg && ws ? (size_t)cfg->workspace_bytes : 0;
    const uint8_t *plan = cfg && cfg->version >= 2 ? static_cast<const uint8_t *>(cfg->plan) : nullptr;
    const PlanLayout pl = plan_layout(A);
    const int32_t *rg_blk = plan ? reinterpret_cast<const int32_t *>(plan + pl.rg_blk) : nullptr;
    if constexpr (sizeof(S) == 4) {
        if (tc_selected(A, engine)) {
            const bool v2 = cfg && cfg->version >= 2;
            const int rc = boo_matmul_tc(A, (const float *)X, (float *)Y, batch, K, rg0, rg1, ws, ws_bytes,
                                         v2 ? cfg->status : nullptr, cfg ? cfg->wait_us : 0, v2 ? cfg->flags : 0,
                                         engine == SPMM_ENGINE_TENSOR_CORES_TF32, plan, s);
            if (rc != SPMM_EUNSUPPORTED || engine >= SPMM_ENGINE_TENSOR_CORES) return rc;
        }
    } else {
        if (engine >= SPMM_ENGINE_TENSOR_CORES) return SPMM_EUNSUPPORTED;
    }
    BooParams<S> p;
    p.rows = A->rows;
    p.cols = A->cols;
    p.K = K;
    p.batch = batch;
    p.nb = A->nb;
    p.tail_nnz = A->tail_nnz;
    p.row_grp_ptr = A->row_grp_ptr;
    p.row_ids = A->row_ids;
    p.col_grp_ptr = A->col_grp_ptr;
    p.col_ids = A->col_ids;
    p.blk_row_grp = A->blk_row_grp;
    p.blk_col_grp = A->blk_col_grp;
    p.blk_nz_ptr = A->blk_nz_ptr;
    p.blk_shift = A->blk_shift;
    p.nz_idx = A->nz_idx;
    p.nz_val = (const S *)A->nz_val;
    p.rem_indptr = A->rem_indptr;
    p.rem_col = A->rem_col_ind;
    p.rem_val = (const S *)A->rem_vals;
    p.tail_row = A->tail_row;
    p.tail_col = A->tail_col;
    p.tail_val = (const S *)A->tail_val;
    p.X = (const S *)X;
    p.Y = (S *)Y;
    p.rowmajor = A->nz_order == SPMM_BOO_ROWMAJOR;
    p.rem_nnz = A->rem_nnz;
    p.n_rg = A->n_rg;
    p.rg_first = 0;
    p.rg_blk = rg_blk;
    p.rgs_per_cta = 1;
    p.nch = 0;
    p.chunk = 0;
    p.chunk_row = nullptr;
    p.part = nullptr;
    const bool aligned = (((uintptr_t)X | (uintptr_t)Y) & 15) == 0;
    // remainder-major matrices: the load-balanced remainder kernels write Y,
    // then the block kernel adds blocks and tail where a row group has any
    p.skip_rem = A->rem_nnz > 0 && 2 * A->rem_nnz >= A->total_nnz;
    if (p.skip_rem && (rg0 != 0 || rg1 != A->n_rg)) return SPMM_EUNSUPPORTED;   // whole matrix only
    if (plan && pl.row_view && pl.short_rows) {
        // a warp per row over the plan's row-ordered copy, rows of groups [rg0, rg1)
        p.rem_indptr = reinterpret_cast<const int32_t *>(plan + pl.rv_ptr);
        p.rem_col = reinterpret_cast<const int32_t *>(plan + pl.rv_col);
        p.rem_val = reinterpret_cast<const S *>(plan + pl.rv_val);
        return row_warp_dispatch<S>(p, rg0, rg1, A->max_nr, reinterpret_cast<const int32_t *>(plan + pl.rv_ident),
                                    aligned, s);
    }
    if (plan && pl.row_view) {
        // the plan's row-ordered copy of every entry: one load-balanced pass writes Y
        p.rem_indptr = reinterpret_cast<const int32_t *>(plan + pl.rv_ptr);
        p.rem_col = reinterpret_cast<const int32_t *>(plan + pl.rv_col);
        p.rem_val = reinterpret_cast<const S *>(plan + pl.rv_val);
        p.rem_nnz = pl.entries;
        const int slab_req = cfg ? cfg->slab_features : 0;
        if (rem_flat_applies(p, aligned, slab_req) &&
            (!ws || ws_bytes < rem_flat_workspace(pl.entries, batch, K, sizeof(S))))
            return SPMM_EWORKSPACE;
        return rem_dispatch<S>(p, aligned, slab_req, ws, s);
    }
    if (p.skip_rem) {
        const int slab_req = cfg ? cfg->slab_features : 0;
        if (rem_flat_applies(p, aligned, slab_req) &&
            (!ws || ws_bytes < rem_flat_workspace(A->rem_nnz, batch, K, sizeof(S))))
            return SPMM_EWORKSPACE;
        const int rc = rem_dispatch<S>(p, aligned, slab_req, ws, s);   // Y = remainder
        if (rc != SPMM_OK) return rc;
    }
    return boo_dispatch<S>(p, rg0, rg1, aligned, s);      // (+)= blocks and tail
}

// Checks shared by the whole-matrix and row-group-range products; then the product.
int boo_matmul_checked(const spmm_boo_dev *A, const void *X, void *Y, int64_t batch, int64_t K, int64_t rg0,
                       int64_t rg1, const spmm_launch_cfg *cfg, cudaStream_t s) {
    if (!A || batch < 0 || K < 0) return SPMM_EINVAL;
    if (cfg && cfg->version != 1 && cfg->version != 2) return SPMM_EINVAL;
    const int engine = cfg ? cfg->engine : SPMM_ENGINE_AUTO;
    if (engine < SPMM_ENGINE_AUTO || engine > SPMM_ENGINE_TENSOR_CORES_TF32) return SPMM_EINVAL;
    if (cfg && cfg->wait_us < 0) return SPMM_EINVAL;
    if (cfg && cfg->version >= 2 && (cfg->flags & ~SPMM_CFG_EXPIRE_FIRST_WAIT)) return SPMM_EINVAL;
    if (cfg && cfg->version >= 2 && (cfg->flags & SPMM_CFG_EXPIRE_FIRST_WAIT) && cfg->wait_us <= 0)
        return SPMM_EINVAL;   // the expiring wait must be short
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return SPMM_EINVAL;
    if (A->nz_order != SPMM_BOO_ROWMAJOR && A->nz_order != SPMM_BOO_COLMAJOR) return SPMM_EINVAL;
    if (A->rows < 0 || A->cols < 0 || A->n_rg < 0 || A->nb < 0 || A->tail_nnz < 0) return SPMM_EINVAL;
    if (rg0 < 0 || rg1 < rg0 || rg1 > A->n_rg) return SPMM_EINVAL;
    if (A->rows > 0x7fffffffLL || A->cols > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    if (A->max_nr > 65536 || A->max_nc > 65536) return SPMM_EUNSUPPORTED;
    if (cfg && cfg->version >= 2 && cfg->status)   // this call's status word starts at 0
        SPMM_CUDA_TRY(cudaMemsetAsync(cfg->status, 0, sizeof(int32_t), s));
    if (batch == 0 || K == 0 || A->rows == 0 || rg0 == rg1) return SPMM_OK;
    if (!Y || (A->cols && !X)) return SPMM_EINVAL;
    if (!A->row_grp_ptr || !A->row_ids || !A->rem_indptr) return SPMM_EINVAL;
    if (A->nb && (!A->blk_row_grp || !A->blk_col_grp || !A->blk_nz_ptr || !A->blk_shift ||
                  !A->nz_idx || !A->nz_val || !A->col_grp_ptr || !A->col_ids))
        return SPMM_EINVAL;
    if (A->n_rg == 0) return SPMM_EINVAL;  // rows > 0 need at least one group
    if (A->scalar_type == SPMM_F32) return boo_matmul_impl<float>(A, X, Y, batch, K, rg0, rg1, engine, cfg, s);
    return boo_matmul_impl<double>(A, X, Y, batch, K, rg0, rg1, engine, cfg, s);
}

}  // namespace
}  // namespace spmm


using namespace spmm;

extern "C" int spmm_boo_matmul(const spmm_boo_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                               const spmm_launch_cfg *cfg, spmm_stream_t stream) {
    return boo_matmul_checked(A, X, Y, batch, K, 0, A ? A->n_rg : 0, cfg, (cudaStream_t)stream);
}

extern "C" int spmm_boo_matmul_groups(const spmm_boo_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                                      int64_t rg_begin, int64_t rg_end, const spmm_launch_cfg *cfg,
                                      spmm_stream_t stream) {
    return boo_matmul_checked(A, X, Y, batch, K, rg_begin, rg_end, cfg, (cudaStream_t)stream);
}

extern "C" size_t spmm_boo_matmul_workspace_size(const spmm_boo_dev *A, int64_t batch, int64_t K,
                                                 const spmm_launch_cfg *cfg) {
    if (!A || batch <= 0 || K <= 0) return 0;
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return 0;
    if (cfg && cfg->version != 1 && cfg->version != 2) return 0;
    if (A->scalar_type == SPMM_F32 && tc_selected(A, cfg ? cfg->engine : SPMM_ENGINE_AUTO)) {
        const size_t w = boo_tc_workspace(A, batch, K);
        if (w || (cfg && cfg->engine >= SPMM_ENGINE_TENSOR_CORES)) return w;
    }
    // remainder-major: the nnz-flat remainder's scratch (16-byte aligned X and Y),
    // over the plan's row-ordered copy of every entry when the plan has one
    const bool rem_major = A->rem_nnz > 0 && 2 * A->rem_nnz >= A->total_nnz;
    const size_t elem = A->scalar_type == SPMM_F32 ? 4 : 8;
    if (!rem_major || (cfg && cfg->slab_features < 0) || K % (int64_t)(16 / elem)) return 0;
    const bool row_view = cfg && cfg->version >= 2 && cfg->plan && plan_row_view(A);
    const int64_t entries = row_view ? A->nnz_c + A->rem_nnz + A->tail_nnz : A->rem_nnz;
    if ((!cfg || cfg->slab_features == 0) && K <= 16 * (int64_t)(16 / elem) && entries <= kShortRow * A->rows)
        return 0;   // half a warp per row, no scratch
    return rem_flat_workspace(entries, batch, K, elem);
}
