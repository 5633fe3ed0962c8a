// spmm_pbr.cu -- Y = A*X for A in PBR format on sm_100a.
//
// Replaces the reference's per-block kernel pbr_spmm_vec_kernel /
// pbr_spmm_zero_idle_kernel plus the concurrent CSR-remainder kernel over a
// memset Y (torch_fast_spdmm/kernels/pbr_kernel.cu:12-326 and 976-1135,
// bindings/bindings_kernels.cu:18-123) with ONE launch: for block-major
// matrices a warp per stripe (pbr_stripe_kernel below), otherwise
// pbr_spmm_kernel, in which each group of LPR lanes owns an output row:
//   * the row's stripe (row / block_rows) has a contiguous run of blocks; the
//     CTA finds the runs of its stripes with one binary search each;
//   * per block the row's bits are (code >> (r % BR) * BC) & mask; the value
//     of bit c is data[offset + popcount(code bits below it)] -- the bit-order
//     consumption of the reference (pbr_matrix.cpp:42-55) -- decoded with
//     __popcll / __ffsll, no bitset scan of the whole code;
//   * then the row's remainder entries; Y is stored once (no memset, no
//     atomics) and is correct for every K (the reference's vec kernel needs K
//     to be a power-of-two multiple of its tile, pbr_kernel.cu:81-87).
#include "spmm_common.cuh"

namespace spmm {
namespace {

constexpr int kPbrThreads = 256;
constexpr int kPbrRows = 32;   // rows per CTA

template <typename S, typename I>
struct PbrParams {
    int64_t rows, cols, K, batch, nb, br, bc;
    const uint64_t *codes;
    const I *coords, *offsets, *rem_indptr, *rem_col;
    const S *data, *rem_val;
    const S *X;
    S *Y;
};

template <typename I>
__device__ __forceinline__ int64_t first_block_of_stripe(const I *coords, int64_t nb, int64_t row0) {
    // blocks are grouped by stripe in ascending order; coords[2b] is the
    // block's top row
    int64_t lo = 0, hi = nb;
    while (lo < hi) {
        int64_t mid = (lo + hi) >> 1;
        if ((int64_t)coords[2 * mid] < row0) lo = mid + 1; else hi = mid;
    }
    return lo;
}

template <typename S, int VEC, int VPT, int LPR>
__device__ __forceinline__ void fma_x(Frag<S, VEC> (&acc)[VPT], S a, const S *xr, const bool (&vm)[VPT]) {
#pragma unroll
    for (int v = 0; v < VPT; ++v)
        if (vm[v]) {
            Frag<S, VEC> x = ldg_frag<S, VEC>(xr + v * LPR * VEC);
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[v].v[q] = fma(a, x.v[q], acc[v].v[q]);
        }
}

template <typename S, typename I, int VEC, int VPT, int LPR>
__global__ void __launch_bounds__(kPbrThreads)
pbr_spmm_kernel(const PbrParams<S, I> p) {
    constexpr int NG = kPbrThreads / LPR;
    constexpr int RPG = kPbrRows / NG;
    constexpr int SLAB = LPR * VPT * VEC;
    static_assert(RPG >= 1 && RPG * NG == kPbrRows, "row mapping");
    __shared__ int64_t stripe_blk[kPbrRows + 2];

    const int tid = threadIdx.x;
    const int g = tid / LPR, l = tid % LPR;
    const int64_t row_base = (int64_t)blockIdx.x * kPbrRows;
    const int64_t f0 = (int64_t)blockIdx.y * SLAB + (int64_t)l * VEC;
    bool vm[VPT];
#pragma unroll
    for (int v = 0; v < VPT; ++v) vm[v] = f0 + (int64_t)v * LPR * VEC < p.K;

    // block runs of the stripes this CTA touches
    const int64_t s_first = row_base / p.br;
    int64_t row_last = row_base + kPbrRows - 1;
    if (row_last >= p.rows) row_last = p.rows - 1;
    const int64_t n_str = row_last / p.br - s_first + 1;   // <= kPbrRows
    if (tid <= n_str) stripe_blk[tid] = first_block_of_stripe(p.coords, p.nb, (s_first + tid) * p.br);
    __syncthreads();

    const uint64_t bcmask = p.bc >= 64 ? ~0ull : ((1ull << p.bc) - 1ull);
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        S *yb = p.Y + bt * p.rows * p.K;
#pragma unroll
        for (int i = 0; i < RPG; ++i) {
            const int64_t r = row_base + g + i * NG;
            if (r >= p.rows) continue;
            Frag<S, VEC> acc[VPT];
#pragma unroll
            for (int v = 0; v < VPT; ++v)
#pragma unroll
                for (int q = 0; q < VEC; ++q) acc[v].v[q] = S(0);
            const int64_t si = r / p.br - s_first;
            const int rin = (int)(r % p.br);
            const int sh = rin * (int)p.bc;
            const uint64_t below = sh >= 64 ? ~0ull : ((1ull << sh) - 1ull);
            for (int64_t b = stripe_blk[si]; b < stripe_blk[si + 1]; ++b) {
                const uint64_t code = p.codes[b];
                uint64_t bits = (sh >= 64 ? 0ull : (code >> sh)) & bcmask;
                if (!bits) continue;
                int64_t off = (int64_t)p.offsets[b] + __popcll(code & below);
                const int64_t col0 = (int64_t)p.coords[2 * b + 1];
                while (bits) {
                    const int c = __ffsll((long long)bits) - 1;
                    bits &= bits - 1;
                    if (col0 + c >= p.cols) continue;   // never set by a valid build
                    fma_x<S, VEC, VPT, LPR>(acc, p.data[off++], xl + (col0 + c) * p.K, vm);
                }
            }
            const int64_t j1 = (int64_t)p.rem_indptr[r + 1];
            int64_t j = (int64_t)p.rem_indptr[r];
            for (; j + 2 <= j1; j += 2) {
                const S a0 = p.rem_val[j], a1 = p.rem_val[j + 1];
                const S *x0 = xl + (int64_t)p.rem_col[j] * p.K;
                const S *x1 = xl + (int64_t)p.rem_col[j + 1] * p.K;
                Frag<S, VEC> t0[VPT], t1[VPT];
#pragma unroll
                for (int v = 0; v < VPT; ++v)
                    if (vm[v]) {
                        t0[v] = ldg_frag<S, VEC>(x0 + v * LPR * VEC);
                        t1[v] = ldg_frag<S, VEC>(x1 + v * LPR * VEC);
                    }
#pragma unroll
                for (int v = 0; v < VPT; ++v)
                    if (vm[v])
#pragma unroll
                        for (int q = 0; q < VEC; ++q) {
                            acc[v].v[q] = fma(a0, t0[v].v[q], acc[v].v[q]);
                            acc[v].v[q] = fma(a1, t1[v].v[q], acc[v].v[q]);
                        }
            }
            if (j < j1) fma_x<S, VEC, VPT, LPR>(acc, p.rem_val[j], xl + (int64_t)p.rem_col[j] * p.K, vm);
            S *yr = yb + r * p.K + f0;
#pragma unroll
            for (int v = 0; v < VPT; ++v)
                if (vm[v]) st_frag<S, VEC>(yr + v * LPR * VEC, acc[v]);
        }
    }
}

// Block-major matrices (most entries in blocks, e.g. a mesh stiffness pattern
// in 8 x 8 blocks): a warp owns one stripe of BR rows and a slab of 32 VEC
// features, with the BR rows' sums in registers.  Per block the warp loads
// the block's values once (two coalesced loads, handed out by shuffles in bit
// order -- the reference's consumption order) and one X row per block column
// that has a set bit, instead of one X row per nonzero, into the warp's
// shared-memory slots; then it walks only the set bits, row by row (the row's
// sum stays a register), reading the column's X slot.  Then the BR rows'
// remainder entries; every Y element is stored once.
constexpr int kStripeWarps = 8;

template <typename S, typename I, int VEC, int BR, int BC>
__global__ void __launch_bounds__(32 * kStripeWarps, 3)
pbr_stripe_kernel(const PbrParams<S, I> p) {
    static_assert(BR * BC <= 64 && BR <= 8 && BC <= 8, "block shape");
    __shared__ Frag<S, VEC> xs[kStripeWarps][BC][32];   // per warp: the block's X rows, a lane's slice each
    const int lane = threadIdx.x & 31;
    Frag<S, VEC> (&xw)[BC][32] = xs[threadIdx.x >> 5];
    const int64_t stripe = (int64_t)blockIdx.x * kStripeWarps + (threadIdx.x >> 5);
    const int64_t row0 = stripe * BR;
    if (row0 >= p.rows) return;
    const int64_t f0 = (int64_t)blockIdx.y * 32 * VEC + (int64_t)lane * VEC;
    const bool fm = f0 < p.K;
    // the stripe's block run (blocks grouped by stripe, ascending)
    const int64_t b0 = first_block_of_stripe(p.coords, p.nb, row0);
    const int64_t b1 = first_block_of_stripe(p.coords, p.nb, row0 + BR);
    for (int64_t bt = blockIdx.z; bt < p.batch; bt += gridDim.z) {
        const S *xl = p.X + bt * p.cols * p.K + f0;
        Frag<S, VEC> acc[BR];
#pragma unroll
        for (int r = 0; r < BR; ++r)
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[r].v[q] = S(0);
        // block b's code, first value and first column; its values a lane each
        // (64 at most: two registers); the next block's are fetched while
        // block b's X rows are in flight, so a block costs one load latency
        uint64_t code = 0;
        int64_t col0 = 0;
        S v_lo = S(0), v_hi = S(0);
        if (b0 < b1) {
            code = __ldg(p.codes + b0);
            const int64_t off = (int64_t)__ldg(p.offsets + b0);
            col0 = (int64_t)__ldg(p.coords + 2 * b0 + 1);
            const int n = __popcll(code);
            v_lo = lane < n ? __ldg(p.data + off + lane) : S(0);
            v_hi = lane + 32 < n ? __ldg(p.data + off + 32 + lane) : S(0);
        }
        for (int64_t b = b0; b < b1; ++b) {
            // every used column's X row in flight at once, into the warp's slots
            // (the block's column mask: the OR of its BR row masks)
            uint32_t colmask = 0;
#pragma unroll
            for (int r = 0; r < BR; ++r) colmask |= (uint32_t)(code >> (r * BC));
            colmask &= (1u << BC) - 1u;
            if (col0 + BC > p.cols) colmask &= (1u << (p.cols > col0 ? p.cols - col0 : 0)) - 1u;
            const unsigned used = colmask;
#pragma unroll
            for (int c = 0; c < BC; ++c)
                if (((used >> c) & 1u) && fm) xw[c][lane] = ldg_frag<S, VEC>(xl + (col0 + c) * p.K);
            uint64_t ncode = 0;
            int64_t noff = 0, ncol0 = 0;
            if (b + 1 < b1) {
                ncode = __ldg(p.codes + b + 1);
                noff = (int64_t)__ldg(p.offsets + b + 1);
                ncol0 = (int64_t)__ldg(p.coords + 2 * b + 3);
            }
            __syncwarp();
            // the set bits in order: row r's bits, lowest column first; the
            // value of the k-th set bit is the block's k-th value
            int rank = 0;
#pragma unroll
            for (int r = 0; r < BR; ++r) {
                uint32_t rb = (uint32_t)(code >> (r * BC)) & ((1u << BC) - 1u);
                while (rb) {   // uniform across the warp
                    const int c = __ffs(rb) - 1;
                    rb &= rb - 1u;
                    const S a = __shfl_sync(kFullMask, rank < 32 ? v_lo : v_hi, rank & 31);   // rank is uniform
                    ++rank;
                    if (fm && ((used >> c) & 1u)) {
                        const Frag<S, VEC> x = xw[c][lane];
#pragma unroll
                        for (int q = 0; q < VEC; ++q) acc[r].v[q] = fma(a, x.v[q], acc[r].v[q]);
                    }
                }
            }
            __syncwarp();   // the slots are rewritten by the next block
            if (b + 1 < b1) {
                const int n = __popcll(ncode);
                v_lo = lane < n ? __ldg(p.data + noff + lane) : S(0);
                v_hi = lane + 32 < n ? __ldg(p.data + noff + 32 + lane) : S(0);
            }
            code = ncode;
            col0 = ncol0;
        }
        S *yb = p.Y + bt * p.rows * p.K + f0;
#pragma unroll
        for (int r = 0; r < BR; ++r) {
            const int64_t row = row0 + r;
            if (row >= p.rows) break;
            const int64_t j0 = (int64_t)__ldg(p.rem_indptr + row), j1 = (int64_t)__ldg(p.rem_indptr + row + 1);
            for (int64_t jb = j0; jb < j1; jb += 32) {
                const int64_t j = jb + lane;
                const int64_t cj = j < j1 ? (int64_t)__ldg(p.rem_col + j) : 0;
                const S aj = j < j1 ? __ldg(p.rem_val + j) : S(0);
                const int m = j1 - jb < 32 ? (int)(j1 - jb) : 32;
                int u = 0;
                for (; u + 2 <= m; u += 2) {
                    const int64_t c0 = __shfl_sync(kFullMask, cj, u), c1 = __shfl_sync(kFullMask, cj, u + 1);
                    const S a0 = __shfl_sync(kFullMask, aj, u), a1 = __shfl_sync(kFullMask, aj, u + 1);
                    if (fm) {
                        const Frag<S, VEC> x0 = ldg_frag<S, VEC>(xl + c0 * p.K);
                        const Frag<S, VEC> x1 = ldg_frag<S, VEC>(xl + c1 * p.K);
#pragma unroll
                        for (int q = 0; q < VEC; ++q) {
                            acc[r].v[q] = fma(a0, x0.v[q], acc[r].v[q]);
                            acc[r].v[q] = fma(a1, x1.v[q], acc[r].v[q]);
                        }
                    }
                }
                if (u < m) {
                    const int64_t c0 = __shfl_sync(kFullMask, cj, u);
                    const S a0 = __shfl_sync(kFullMask, aj, u);
                    if (fm) {
                        const Frag<S, VEC> x0 = ldg_frag<S, VEC>(xl + c0 * p.K);
#pragma unroll
                        for (int q = 0; q < VEC; ++q) acc[r].v[q] = fma(a0, x0.v[q], acc[r].v[q]);
                    }
                }
            }
            if (fm) st_frag<S, VEC>(yb + row * p.K, acc[r]);
        }
    }
}

template <typename S, typename I, int VEC, int BR, int BC>
int launch_pbr_stripe(const PbrParams<S, I> &p, cudaStream_t s) {
    const int64_t slabs = ceil_div(p.K, 32 * VEC);
    const int64_t ctas = ceil_div(ceil_div(p.rows, (int64_t)BR), (int64_t)kStripeWarps);
    if (slabs > 65535 || ctas > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    dim3 grid((unsigned)ctas, (unsigned)slabs, (unsigned)(p.batch < 65535 ? p.batch : 65535));
    pbr_stripe_kernel<S, I, VEC, BR, BC><<<grid, 32 * kStripeWarps, 0, s>>>(p);
    SPMM_PRODUCT_LAUNCHED();
    return SPMM_OK;
}

template <typename S, typename I, int VEC, int VPT, int LPR>
int launch_pbr(const PbrParams<S, I> &p, cudaStream_t s) {
    constexpr int SLAB = LPR * VPT * VEC;
    const int64_t slabs = ceil_div(p.K, SLAB);
    const int64_t ctas = ceil_div(p.rows, kPbrRows);
    if (slabs > 65535 || ctas > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    dim3 grid((unsigned)ctas, (unsigned)slabs, (unsigned)(p.batch < 65535 ? p.batch : 65535));
    pbr_spmm_kernel<S, I, VEC, VPT, LPR><<<grid, kPbrThreads, 0, s>>>(p);
    SPMM_PRODUCT_LAUNCHED();
    return SPMM_OK;
}

template <typename S, typename I>
int pbr_dispatch(const PbrParams<S, I> &p, bool aligned, bool block_major, cudaStream_t s) {
    const int64_t K = p.K;
    constexpr int V = sizeof(S) == 4 ? 4 : 2;
    // block-major matrices with at least one full warp slab of features: a
    // warp per stripe (the reference's launchable shapes 2x2, 4x4, 8x8)
    if (aligned && K % V == 0 && K >= 32 * V && block_major && p.br == p.bc) {
        if (p.br == 8) return launch_pbr_stripe<S, I, V, 8, 8>(p, s);
        if (p.br == 4) return launch_pbr_stripe<S, I, V, 4, 4>(p, s);
        if (p.br == 2) return launch_pbr_stripe<S, I, V, 2, 2>(p, s);
    }
    if (aligned && K % V == 0) {
        if (K <= 8 * V) return launch_pbr<S, I, V, 1, 8>(p, s);
        if (K <= 16 * V) return launch_pbr<S, I, V, 1, 16>(p, s);
        if (K <= 32 * V) return launch_pbr<S, I, V, 1, 32>(p, s);
        if (K <= 64 * V) return launch_pbr<S, I, V, 2, 32>(p, s);
        return launch_pbr<S, I, V, 4, 32>(p, s);
    }
    if (K <= 32) return launch_pbr<S, I, 1, 1, 32>(p, s);
    if (K <= 64) return launch_pbr<S, I, 1, 2, 32>(p, s);
    return launch_pbr<S, I, 1, 4, 32>(p, s);
}

template <typename S, typename I>
int pbr_matmul_impl(const spmm_pbr_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                    cudaStream_t s) {
    PbrParams<S, I> p;
    p.rows = A->rows;
    p.cols = A->cols;
    p.K = K;
    p.batch = batch;
    p.nb = A->nb;
    p.br = A->block_rows;
    p.bc = A->block_cols;
    p.codes = A->codes;
    p.coords = (const I *)A->coords;
    p.offsets = (const I *)A->offsets;
    p.rem_indptr = (const I *)A->rem_indptr;
    p.rem_col = (const I *)A->rem_col_ind;
    p.data = (const S *)A->data;
    p.rem_val = (const S *)A->rem_vals;
    p.X = (const S *)X;
    p.Y = (S *)Y;
    const uintptr_t mis = ((uintptr_t)X | (uintptr_t)Y) & 15;
    return pbr_dispatch<S, I>(p, mis == 0, 2 * A->nnz_c >= A->nnz_c + A->rem_nnz, s);
}

}  // namespace
}  // namespace spmm

using namespace spmm;

extern "C" int spmm_pbr_matmul(const spmm_pbr_dev *A, const void *X, void *Y, int64_t batch, int64_t K,
                               const spmm_launch_cfg *cfg, spmm_stream_t stream) {
    if (!A || batch < 0 || K < 0) return SPMM_EINVAL;
    if (cfg && cfg->version != 1 && cfg->version != 2) return SPMM_EINVAL;
    if (A->scalar_type != SPMM_F32 && A->scalar_type != SPMM_F64) return SPMM_EINVAL;
    if (A->index_type != SPMM_INDEX_I32 && A->index_type != SPMM_INDEX_I64) return SPMM_EINVAL;
    if (A->rows < 0 || A->cols < 0 || A->nb < 0) return SPMM_EINVAL;
    if (A->block_rows <= 0 || A->block_cols <= 0 || A->block_rows * A->block_cols > 64)
        return SPMM_EINVAL;
    // no bounded waits in the PBR kernel: its status word (if any) ends at 0
    if (cfg && cfg->version >= 2 && cfg->status)
        if (cudaMemsetAsync(cfg->status, 0, sizeof(int32_t), (cudaStream_t)stream) != cudaSuccess) return SPMM_ECUDA;
    if (batch == 0 || K == 0 || A->rows == 0) return SPMM_OK;
    if (!Y || (A->cols && !X) || !A->rem_indptr) return SPMM_EINVAL;
    if (A->nb && (!A->codes || !A->coords || !A->offsets || !A->data)) return SPMM_EINVAL;
    cudaStream_t s = (cudaStream_t)stream;
    if (A->scalar_type == SPMM_F32) {
        if (A->index_type == SPMM_INDEX_I32) return pbr_matmul_impl<float, int32_t>(A, X, Y, batch, K, s);
        return pbr_matmul_impl<float, int64_t>(A, X, Y, batch, K, s);
    }
    if (A->index_type == SPMM_INDEX_I32) return pbr_matmul_impl<double, int32_t>(A, X, Y, batch, K, s);
    return pbr_matmul_impl<double, int64_t>(A, X, Y, batch, K, s);
}
