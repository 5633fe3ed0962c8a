// hem.cu -- multilevel heavy-edge matching (HEM) labels on the GPU, the
// reference's default BOO clustering (torch_fast_spdmm/torch_fast_spdmm/
// clustering.py:128-351), with the same result as its host restatement.
//
// Per level, on the binary pattern P of the current (contracted) rows:
//   * similarity graph (clustering.py:128-185): columns of degree above
//     hub_degree are dropped; w(i, j) = shared columns of rows i != j.  Every
//     (i, j) incidence is generated for a chunk of rows, radix-sorted and
//     run-length counted; a second sort by (i, -w, j) keeps each row's topk
//     heaviest (ties by column); the directed lists are united over both
//     directions (w is symmetric, so max(G, G^T) is the union);
//   * up to residual_rounds matching rounds (:188-268): each active vertex
//     picks its best live edge by (w desc, pair hash desc, column asc);
//     mutual picks whose merge respects the size / nnz caps are merged;
//   * contraction (:271-351): new rows are the unions of the matched pairs'
//     column sets (rows in index order of their smaller member); the loop
//     ends when a level matches nothing.
// Everything is integer arithmetic with the reference's tie-breaks, so the
// labels are identical.  Scratch comes from the stream-ordered allocator.
#include <algorithm>
#include <utility>
#include <vector>

#include "common.cuh"

namespace spmm {
namespace {

constexpr int kHemThreads = 256;
constexpr int64_t kPairBudget = 1ll << 27;   // (i, j) incidences sorted per chunk

template <typename T>
struct DBuf {
    T *p = nullptr;
    cudaStream_t s = nullptr;
    DBuf() = default;
    DBuf(const DBuf &) = delete;
    DBuf &operator=(const DBuf &) = delete;
    int alloc(int64_t n, cudaStream_t st) {
        release();
        s = st;
        return cudaMallocAsync(&p, (size_t)(n > 0 ? n : 1) * sizeof(T), st) == cudaSuccess ? SPMM_OK : SPMM_ECUDA;
    }
    void release() {
        if (p) cudaFreeAsync(p, s);
        p = nullptr;
    }
    ~DBuf() { release(); }
};

template <typename T>
int to_host(T *dst, const T *src, int64_t n, cudaStream_t s) {
    if (n <= 0) return SPMM_OK;
    SPMM_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)n * sizeof(T), cudaMemcpyDeviceToHost, s));
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    return SPMM_OK;
}

inline unsigned warps_grid(int64_t rows) { return grid_for(rows * 32, kHemThreads); }

// Symmetric 63-bit hash of the unordered pair {a, b} (a splitmix64 mix of the
// ordered pair (min, max)); the same function as the host restatement.
__device__ __forceinline__ uint64_t pair_hash(int64_t a, int64_t b) {
    const uint64_t lo = (uint64_t)(a < b ? a : b), hi = (uint64_t)(a < b ? b : a);
    uint64_t h = (lo * 0x9E3779B97F4A7C15ull) ^ (hi * 0xC2B2AE3D27D4EB4Full);
    h ^= h >> 30;
    h *= 0xBF58476D1CE4E5B9ull;
    h ^= h >> 27;
    h *= 0x94D049BB133111EBull;
    h ^= h >> 31;
    return h >> 1;
}

__global__ void col_deg_kernel(const int32_t *__restrict__ idx, int64_t nnz, uint32_t *__restrict__ deg) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nnz; k += (int64_t)gridDim.x * blockDim.x)
        atomicAdd(deg + idx[k], 1u);
}

// Warp per row: kept entries (column degree <= hub) -- count (out == null) or
// emit in order; also the row's incidence count (sum of kept column degrees).
__global__ void prune_kernel(const int64_t *__restrict__ ptr, const int32_t *__restrict__ idx, int64_t n,
                             const uint32_t *__restrict__ deg, uint32_t hub, int64_t *__restrict__ cnt,
                             int64_t *__restrict__ pairs, const int64_t *__restrict__ optr,
                             int32_t *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; r < n; r += nw) {
        const int64_t e0 = ptr[r], e1 = ptr[r + 1];
        int64_t kept = 0, inc = 0;
        int64_t o = out ? optr[r] : 0;
        for (int64_t b = e0; b < e1; b += 32) {
            const int64_t k = b + lane;
            const int32_t c = k < e1 ? idx[k] : 0;
            const uint32_t d = k < e1 ? deg[c] : 0u;
            const bool keep = k < e1 && d <= hub;
            const unsigned m = __ballot_sync(kFullMask, keep);
            if (out && keep) out[o + __popc(m & lanemask_lt())] = c;
            o += __popc(m);
            kept += __popc(m);
            uint64_t s = keep ? d : 0u;
#pragma unroll
            for (int w = 16; w > 0; w >>= 1) s += __shfl_xor_sync(kFullMask, s, w);
            inc += (int64_t)s;
        }
        if (lane == 0 && !out) {
            cnt[r] = kept;
            pairs[r] = inc;
        }
    }
}

// Column-major copy of the pruned pattern: rows of each kept column.
__global__ void transpose_kernel(const int64_t *__restrict__ ptr, const int32_t *__restrict__ idx, int64_t n,
                                 const int64_t *__restrict__ tptr, uint32_t *__restrict__ tcur,
                                 int32_t *__restrict__ trow) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; r < n; r += nw)
        for (int64_t k = ptr[r] + lane; k < ptr[r + 1]; k += 32) {
            const int32_t c = idx[k];
            trow[tptr[c] + atomicAdd(tcur + c, 1u)] = (int32_t)r;
        }
}

// Warp per listed row b (row i = list[b]): every incidence (i, j) through a
// kept column as key b << jb | j at start[b] - start[0] on; j == i becomes the
// all-ones sentinel (sorts last).
__global__ void gen_pairs_kernel(const int64_t *__restrict__ ptr, const int32_t *__restrict__ idx,
                                 const int64_t *__restrict__ tptr, const int32_t *__restrict__ trow,
                                 const int64_t *__restrict__ list, const int64_t *__restrict__ start, int64_t rows,
                                 int jb, uint64_t sentinel, uint64_t *__restrict__ keys) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; b < rows; b += nw) {
        const int64_t i = list[b];
        int64_t o = start[b] - start[0];
        for (int64_t k = ptr[i]; k < ptr[i + 1]; ++k) {
            const int32_t c = idx[k];
            const int64_t t0 = tptr[c], t1 = tptr[c + 1];
            for (int64_t t = t0 + lane; t < t1; t += 32) {
                const int64_t j = trow[t];
                keys[o + (t - t0)] = j == i ? sentinel : ((uint64_t)b << jb) | (uint64_t)j;
            }
            o += t1 - t0;
        }
    }
}

// Run heads of the sorted keys (sentinels excluded): flag 1 at a new key.
__global__ void head_flags_kernel(const uint64_t *__restrict__ keys, int64_t n, uint64_t sentinel,
                                  int64_t *__restrict__ flag) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
        flag[k] = keys[k] != sentinel && (k == 0 || keys[k] != keys[k - 1]) ? 1 : 0;
}

// Unique (i, j) with its count w, re-keyed (i << (wb + jb)) | (wmax - w) << jb | j
// so one ascending sort orders each row by (w desc, j asc).
__global__ void rle_kernel(const uint64_t *__restrict__ keys, int64_t n, uint64_t sentinel,
                           const int64_t *__restrict__ pos, int jb, int wb, uint64_t *__restrict__ out) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t key = keys[k];
        if (key == sentinel || (k > 0 && key == keys[k - 1])) continue;
        int64_t e = k + 1;
        while (e < n && keys[e] == key) ++e;
        const uint64_t w = (uint64_t)(e - k);
        const uint64_t il = key >> jb, j = key & ((1ull << jb) - 1ull);
        const uint64_t wmax = (1ull << wb) - 1ull;
        out[pos[k]] = (il << (wb + jb)) | ((wmax - (w < wmax ? w : wmax)) << jb) | j;
    }
}

// Sorted (row, -w, j) keys -> each row's first topk as directed edges (i, j, w).
__global__ void topk_flags_kernel(const uint64_t *__restrict__ keys, int64_t n, int jb, int wb, int64_t topk,
                                  int64_t *__restrict__ flag) {
    const int sh = wb + jb;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t row = keys[k] >> sh;
        bool keep = true;
        if (topk >= 0) {
            // the row's first topk entries: the entry topk places back is of another row
            keep = k < topk || (keys[k - topk] >> sh) != row;
        }
        flag[k] = keep ? 1 : 0;
    }
}

__global__ void topk_emit_kernel(const uint64_t *__restrict__ keys, int64_t n, const int64_t *__restrict__ flag,
                                 const int64_t *__restrict__ pos, const int64_t *__restrict__ list, int jb, int wb,
                                 int64_t ebase, uint64_t *__restrict__ ekey, uint32_t *__restrict__ ew) {
    const int sh = wb + jb;
    const uint64_t wmax = (1ull << wb) - 1ull, jm = (1ull << jb) - 1ull;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        if (!flag[k]) continue;
        const uint64_t key = keys[k];
        const uint64_t i = (uint64_t)list[key >> sh], j = key & jm;
        const uint32_t w = (uint32_t)(wmax - ((key >> jb) & wmax));
        const int64_t o = ebase + 2 * pos[k];
        ekey[o] = (i << jb) | j;   // both directions; equal pairs collapse after the sort
        ekey[o + 1] = (j << jb) | i;
        ew[o] = w;
        ew[o + 1] = w;
    }
}

// Sorted directed edge keys -> symmetric graph CSR (duplicates dropped).
__global__ void edge_heads_kernel(const uint64_t *__restrict__ key, int64_t n, int64_t *__restrict__ flag,
                                  int jb, unsigned long long *__restrict__ rowcnt) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        const bool head = k == 0 || key[k] != key[k - 1];
        flag[k] = head ? 1 : 0;
        if (head) atomicAdd(rowcnt + (key[k] >> jb), 1ull);
    }
}

__global__ void edge_emit_kernel(const uint64_t *__restrict__ key, const uint32_t *__restrict__ w, int64_t n,
                                 const int64_t *__restrict__ flag, const int64_t *__restrict__ pos, int jb,
                                 int32_t *__restrict__ gcol, uint32_t *__restrict__ gw) {
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
        if (!flag[k]) continue;
        gcol[pos[k]] = (int32_t)(key[k] & ((1ull << jb) - 1ull));
        gw[pos[k]] = w[k];
    }
}

struct Caps {
    int64_t max_size, max_nnz;   // < 0: none
    __device__ __forceinline__ bool ok(const int64_t *size, const int64_t *nnz, int64_t a, int64_t b) const {
        return (max_size < 0 || size[a] + size[b] <= max_size) && (max_nnz < 0 || nnz[a] + nnz[b] <= max_nnz);
    }
};

// Edge order of the pick: (w desc, pair hash desc, column asc); c < 0 is "none".
__device__ __forceinline__ bool better_edge(uint32_t w, uint64_t h, int64_t c, uint32_t bw, uint64_t bh, int64_t bc) {
    return c >= 0 && (bc < 0 || w > bw || (w == bw && (h > bh || (h == bh && c < bc))));
}

// This thread's best over the edges [e0, e1) of vertex r, stepping by `step`.
__device__ __forceinline__ void best_over(const int32_t *__restrict__ gcol, const uint32_t *__restrict__ gw,
                                          int64_t r, int64_t e0, int64_t e1, int64_t step,
                                          const uint8_t *__restrict__ active, const int64_t *__restrict__ size,
                                          const int64_t *__restrict__ nnz, const Caps &caps, int feasible_first,
                                          uint32_t &bw, uint64_t &bh, int64_t &bc) {
    for (int64_t e = e0; e < e1; e += step) {
        const int64_t c = gcol[e];
        if (!active[c] || (feasible_first && !caps.ok(size, nnz, r, c))) continue;
        const uint32_t w = gw[e];
        const uint64_t h = pair_hash(r, c);
        if (better_edge(w, h, c, bw, bh, bc)) {
            bw = w;
            bh = h;
            bc = c;
        }
    }
}

__device__ __forceinline__ void warp_best(uint32_t &bw, uint64_t &bh, int64_t &bc) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint32_t ow = __shfl_xor_sync(kFullMask, bw, o);
        const uint64_t oh = __shfl_xor_sync(kFullMask, bh, o);
        const int64_t oc = __shfl_xor_sync(kFullMask, bc, o);
        if (better_edge(ow, oh, oc, bw, bh, bc)) {
            bw = ow;
            bh = oh;
            bc = oc;
        }
    }
}

// Vertices of more than kHeavyEdges edges (vertices that many rows keep among
// their top k) are picked by a CTA each (best_heavy_kernel); a warp per
// vertex takes the rest.
constexpr int64_t kHeavyEdges = 4096;
constexpr int kHeavyThreads = 512;

// Warp per vertex: its best live edge by (w desc, hash desc, column asc).
__global__ void best_kernel(const unsigned long long *__restrict__ gptr, const int32_t *__restrict__ gcol,
                            const uint32_t *__restrict__ gw, int64_t n, const uint8_t *__restrict__ active,
                            const int64_t *__restrict__ size, const int64_t *__restrict__ nnz, Caps caps,
                            int feasible_first, int64_t *__restrict__ best) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; r < n; r += nw) {
        const int64_t e0 = (int64_t)gptr[r], e1 = (int64_t)gptr[r + 1];
        if (e1 - e0 > kHeavyEdges) continue;   // best_heavy_kernel's vertex
        uint32_t bw = 0;
        uint64_t bh = 0;
        int64_t bc = -1;
        if (active[r]) best_over(gcol, gw, r, e0 + lane, e1, 32, active, size, nnz, caps, feasible_first, bw, bh, bc);
        warp_best(bw, bh, bc);
        if (lane == 0) best[r] = bc;
    }
}

// Vertices of the level graph with more than kHeavyEdges edges, in any order.
__global__ void heavy_list_kernel(const unsigned long long *__restrict__ gptr, int64_t n,
                                  unsigned long long *__restrict__ count, int64_t *__restrict__ list) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        if ((int64_t)(gptr[r + 1] - gptr[r]) > kHeavyEdges) list[atomicAdd(count, 1ull)] = r;
}

// CTA per heavy vertex: the same pick as best_kernel.
__global__ void __launch_bounds__(kHeavyThreads) best_heavy_kernel(
    const unsigned long long *__restrict__ gptr, const int32_t *__restrict__ gcol, const uint32_t *__restrict__ gw,
    const int64_t *__restrict__ list, int64_t n_heavy, const uint8_t *__restrict__ active,
    const int64_t *__restrict__ size, const int64_t *__restrict__ nnz, Caps caps, int feasible_first,
    int64_t *__restrict__ best) {
    __shared__ uint32_t sw[kHeavyThreads / 32];
    __shared__ uint64_t sh[kHeavyThreads / 32];
    __shared__ int64_t sc[kHeavyThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t v = blockIdx.x; v < n_heavy; v += gridDim.x) {
        const int64_t r = list[v];
        uint32_t bw = 0;
        uint64_t bh = 0;
        int64_t bc = -1;
        if (active[r])
            best_over(gcol, gw, r, (int64_t)gptr[r] + threadIdx.x, (int64_t)gptr[r + 1], kHeavyThreads, active, size,
                      nnz, caps, feasible_first, bw, bh, bc);
        warp_best(bw, bh, bc);
        __syncthreads();   // the previous vertex's reduction has been read
        if (lane == 0) {
            sw[warp] = bw;
            sh[warp] = bh;
            sc[warp] = bc;
        }
        __syncthreads();
        if (warp == 0) {
            bw = lane < kHeavyThreads / 32 ? sw[lane] : 0u;
            bh = lane < kHeavyThreads / 32 ? sh[lane] : 0ull;
            bc = lane < kHeavyThreads / 32 ? sc[lane] : -1;
            warp_best(bw, bh, bc);
            if (lane == 0) best[r] = bc;
        }
    }
}

// Mutual picks (r < best[r]) that respect the caps: matched, deactivated.
__global__ void mutual_kernel(const int64_t *__restrict__ best, int64_t n, const int64_t *__restrict__ size,
                              const int64_t *__restrict__ nnz, Caps caps, int64_t *__restrict__ mate,
                              uint8_t *__restrict__ active, unsigned long long *__restrict__ matched) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = best[r];
        if (b > r && best[b] == r && caps.ok(size, nnz, r, b)) {
            mate[r] = b;
            mate[b] = r;
            active[r] = 0;
            active[b] = 0;
            atomicAdd(matched, 1ull);
        }
    }
}

// 1 for vertices that stay a row of the next level (not the larger member of a pair).
__global__ void root_flags_kernel(const int64_t *__restrict__ mate, int64_t n, int64_t *__restrict__ flag) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x)
        flag[r] = (mate[r] >= 0 && mate[r] < r) ? 0 : 1;
}

// lower_bound of x in the sorted run a[0, n).
__device__ __forceinline__ int64_t lower_bound_run(const int32_t *__restrict__ a, int64_t n, int32_t x) {
    int64_t lo = 0, hi = n;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (a[mid] < x) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// Warp per vertex: new_id of every vertex; sizes / nnz summed into the new
// rows; the new pattern's row lengths (a matched pair: |A u B| = |A| + |B|
// minus the entries of B found in A, one binary search per entry of B).
__global__ void contract_kernel(const int64_t *__restrict__ mate, int64_t n, const int64_t *__restrict__ rank,
                                const int64_t *__restrict__ size, const int64_t *__restrict__ nnz,
                                const int64_t *__restrict__ ptr, const int32_t *__restrict__ idx,
                                int64_t *__restrict__ new_id, unsigned long long *__restrict__ nsize,
                                unsigned long long *__restrict__ nnnz, int64_t *__restrict__ nlen) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; r < n; r += nw) {
        const int64_t m = mate[r];
        const int64_t root = (m >= 0 && m < r) ? m : r;
        const int64_t id = rank[root];
        if (lane == 0) {
            new_id[r] = id;
            atomicAdd(nsize + id, (unsigned long long)size[r]);
            atomicAdd(nnnz + id, (unsigned long long)nnz[r]);
        }
        if (root != r) continue;
        const int64_t la = ptr[r + 1] - ptr[r];
        int64_t len = la;
        if (m > r) {
            const int32_t *A = idx + ptr[r], *B = idx + ptr[m];
            const int64_t lb = ptr[m + 1] - ptr[m];
            int64_t dup = 0;
            for (int64_t j = lane; j < lb; j += 32) {
                const int64_t p = lower_bound_run(A, la, B[j]);
                dup += p < la && A[p] == B[j];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dup += __shfl_xor_sync(kFullMask, dup, o);
            len = la + lb - dup;
        }
        if (lane == 0) nlen[id] = len;
    }
}

// Warp per new row: its sorted column list.  An unmatched row is copied; a
// pair's union places A's entry i at i + (B entries below it that are not in
// A) and B's entries missing from A at (their rank among those) + (A entries
// below them), each found by a binary search, the ranks by warp ballots.
__global__ void contract_emit_kernel(const int64_t *__restrict__ mate, int64_t n, const int64_t *__restrict__ rank,
                                     const int64_t *__restrict__ ptr, const int32_t *__restrict__ idx,
                                     const int64_t *__restrict__ nptr, int32_t *__restrict__ nidx) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * (blockDim.x / 32);
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / 32; r < n; r += nw) {
        const int64_t m = mate[r];
        if (m >= 0 && m < r) continue;
        int32_t *out = nidx + nptr[rank[r]];
        const int32_t *A = idx + ptr[r];
        const int64_t la = ptr[r + 1] - ptr[r];
        if (m < 0) {
            for (int64_t i = lane; i < la; i += 32) out[i] = A[i];
            continue;
        }
        const int32_t *B = idx + ptr[m];
        const int64_t lb = ptr[m + 1] - ptr[m];
        int64_t common = 0;   // A entries below the current chunk that are in B
        for (int64_t i0 = 0; i0 < la; i0 += 32) {
            const int64_t i = i0 + lane;
            int64_t p = 0;
            bool in_b = false;
            if (i < la) {
                p = lower_bound_run(B, lb, A[i]);
                in_b = p < lb && B[p] == A[i];
            }
            const unsigned mask = __ballot_sync(kFullMask, in_b);
            if (i < la) out[i + p - (common + __popc(mask & lanemask_lt()))] = A[i];
            common += __popc(mask);
        }
        int64_t missing = 0;  // B entries below the current chunk that are not in A
        for (int64_t j0 = 0; j0 < lb; j0 += 32) {
            const int64_t j = j0 + lane;
            int64_t q = 0;
            bool out_a = false;
            if (j < lb) {
                q = lower_bound_run(A, la, B[j]);
                out_a = !(q < la && A[q] == B[j]);
            }
            const unsigned mask = __ballot_sync(kFullMask, out_a);
            if (out_a) out[missing + __popc(mask & lanemask_lt()) + q] = B[j];
            missing += __popc(mask);
        }
    }
}

__global__ void relabel_kernel(int64_t *__restrict__ labels, int64_t n, const int64_t *__restrict__ new_id) {
    for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n; v += (int64_t)gridDim.x * blockDim.x)
        labels[v] = new_id[labels[v]];
}

template <typename T>
__global__ void copy_cast_kernel(const unsigned long long *__restrict__ in, T *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (T)in[i];
}

__global__ void iota64_kernel(int64_t *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = i;
}

__global__ void fill_kernel(int64_t *__restrict__ out, int64_t n, int64_t v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = v;
}

__global__ void widen_kernel(const uint32_t *__restrict__ in, int64_t *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = in[i];
}

__global__ void diff_kernel(const int64_t *__restrict__ ptr, int64_t n, int64_t *__restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = ptr[i + 1] - ptr[i];
}

// ---- per-row counting by hashing (top-k > 0) ----
//
// A CTA per row: the row's incidences are counted in an open-addressing
// table (shared memory, or a global region for rows whose table would not
// fit), then the row's topk entries by (w desc, j asc) are found by a radix
// select on the key (wmax - w) << jb | j (unique per row) and emitted as both
// directions of the directed edge.  No sort of the incidences is needed.
constexpr int kHashThreads = 256;
constexpr int kTinySlots = 4096;    // most rows: 32 KB of (key, count) slots, more CTAs per SM
constexpr int kSmemSlots = 8192;    // small rows: 64 KB, 3 CTAs per SM
constexpr int kMidSlots = 16384;    // mid rows: 128 KB, one CTA of 512 threads per SM

// Tables of (class_lo(SLOTS), SLOTS] slots are counted by the launch of SLOTS
// (0: the global-memory class, above kMidSlots).
__host__ __device__ constexpr int64_t class_lo(int slots) {
    return slots == kTinySlots ? 0 : slots == kSmemSlots ? kTinySlots : slots == kMidSlots ? kSmemSlots : kMidSlots;
}

// Slots of a row's table: a power of two, at least 64 and twice the row's incidences (0: no table).
inline int64_t table_slots(int64_t inc) {
    if (inc <= 1) return 0;
    int64_t S = 64;
    while (S < 2 * inc) S <<= 1;
    return S;
}

__device__ __forceinline__ uint32_t slot_of(uint32_t j, int lg) {
    return lg ? (j * 0x9E3779B1u) >> (32 - lg) : 0u;
}

// SLOTS: the shared-memory table of this launch's rows (tables of up to SLOTS
// and more than SLOTS / 2 slots, the smallest class from 64); 0: rows whose
// table exceeds kMidSlots, in global memory.
struct SelectSmem {
    uint32_t hist[256];
    unsigned long long red_u, red_w, sel_prefix;
    long long sel_k;
};

// Over the slots [0, S) of a counted table (key >= 0: occupied): U = the
// occupied slots, W = the heaviest count and kth = the topk-th smallest key
// (W - w) << jb | j (~0 when U <= topk: every entry kept), by a radix select
// a byte at a time.  Every thread of the CTA calls it after a barrier and gets
// the same three values.
template <int THREADS>
__device__ void count_and_select(const int32_t *key, const uint32_t *cnt, int64_t S, int jb, long long topk,
                                 SelectSmem &sm, unsigned long long &U, unsigned long long &W,
                                 unsigned long long &kth) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        sm.red_u = 0;
        sm.red_w = 0;
    }
    __syncthreads();
    unsigned long long u = 0, wm = 0;
    for (int64_t t = tid; t < S; t += THREADS)
        if (key[t] >= 0) {
            ++u;
            wm = cnt[t] > wm ? cnt[t] : wm;
        }
    atomicAdd(&sm.red_u, u);
    atomicMax(&sm.red_w, wm);
    __syncthreads();
    U = sm.red_u;
    W = sm.red_w;
    kth = ~0ull;
    if ((long long)U <= topk) return;
    const int bits = jb + (64 - __clzll((long long)W));   // key (W - w) << jb | j
    if (tid == 0) {
        sm.sel_prefix = 0;
        sm.sel_k = topk;
    }
    unsigned long long mask = 0;
    for (int shift = ((bits + 7) / 8 - 1) * 8; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += THREADS) sm.hist[b] = 0;
        __syncthreads();
        const unsigned long long prefix = sm.sel_prefix;
        for (int64_t t = tid; t < S; t += THREADS) {
            if (key[t] < 0) continue;
            const unsigned long long K = ((W - cnt[t]) << jb) | (unsigned long long)key[t];
            if ((K & mask) == prefix) atomicAdd(&sm.hist[(K >> shift) & 255], 1u);
        }
        __syncthreads();
        if (warp == 0) {
            // the first byte value v whose running count reaches k (255 when
            // none before it does): lanes own 8 bins each, one warp scan
            const long long k = sm.sel_k;
            unsigned c[8];
            long long own = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                c[q] = sm.hist[lane * 8 + q];
                own += c[q];
            }
            long long incl = own;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const long long up = __shfl_up_sync(kFullMask, incl, o);
                if (lane >= o) incl += up;
            }
            long long cum = incl - own;
            if (cum < k && (k <= incl || lane == 31)) {
                int v = lane * 8;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (v == 255 || cum + c[q] >= k) break;
                    cum += c[q];
                    ++v;
                }
                sm.sel_k = k - cum;
                sm.sel_prefix = prefix | ((unsigned long long)v << shift);
            }
        }
        mask |= 255ull << shift;
        __syncthreads();
    }
    kth = sm.sel_prefix;
}

__device__ __forceinline__ void emit_edge(int64_t i, int32_t j, uint32_t w, int jb,
                                          unsigned long long *__restrict__ ecount, uint64_t *__restrict__ ekey,
                                          uint32_t *__restrict__ ew) {
    const unsigned long long o = atomicAdd(ecount, 2ull);
    ekey[o] = ((uint64_t)i << jb) | (uint64_t)j;
    ekey[o + 1] = ((uint64_t)j << jb) | (uint64_t)i;
    ew[o] = w;
    ew[o + 1] = w;
}

template <int THREADS, int SLOTS>
__global__ void __launch_bounds__(THREADS) hash_topk_kernel(
    const int64_t *__restrict__ ptr, const int32_t *__restrict__ idx, const int64_t *__restrict__ tptr,
    const int32_t *__restrict__ trow, const int64_t *__restrict__ pinc, const int64_t *__restrict__ goff,
    int32_t *__restrict__ gkey, uint32_t *__restrict__ gcnt, int64_t n, int jb, int64_t topk,
    unsigned long long *__restrict__ ecount, uint64_t *__restrict__ ekey, uint32_t *__restrict__ ew) {
    extern __shared__ uint32_t hsm[];
    int32_t *skey = reinterpret_cast<int32_t *>(hsm);
    uint32_t *scnt = hsm + (SLOTS > 0 ? SLOTS : 1);
    __shared__ SelectSmem sm;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int64_t i = blockIdx.x; i < n; i += gridDim.x) {
        const int64_t inc = pinc[i];
        if (inc <= 1) continue;   // only itself (or nothing): no candidates
        int lg = 6;
        while ((1ll << lg) < 2 * inc) ++lg;
        const int64_t S = 1ll << lg;
        const int64_t hi_cap = SLOTS == 0 ? INT64_MAX : SLOTS;
        if (S <= class_lo(SLOTS) || S > hi_cap) continue;   // another launch's rows
        int32_t *key = skey;
        uint32_t *cnt = scnt;
        if (SLOTS == 0) {   // the row's region of the global tables
            key = gkey + goff[i];
            cnt = gcnt + goff[i];
        }
        __syncthreads();   // the previous row is done with the table
        for (int64_t t = tid; t < S; t += THREADS) {
            key[t] = -1;
            cnt[t] = 0;
        }
        __syncthreads();
        // insert: warps take the row's columns, lanes the column's rows
        for (int64_t k = ptr[i] + warp; k < ptr[i + 1]; k += THREADS / 32) {
            const int32_t c = idx[k];
            for (int64_t t = tptr[c] + lane; t < tptr[c + 1]; t += 32) {
                const int32_t j = trow[t];
                if (j == i) continue;
                uint32_t h = slot_of((uint32_t)j, lg);
                for (;;) {
                    const int32_t prev = atomicCAS(key + h, -1, j);
                    if (prev == -1 || prev == j) {
                        atomicAdd(cnt + h, 1u);
                        break;
                    }
                    h = (h + 1) & (uint32_t)(S - 1);
                }
            }
        }
        __syncthreads();
        int64_t live = S;   // slots the selection reads
        if (SLOTS == 0) {
            // a global table is at most half full: its occupied slots move to
            // the front (in slot order, a block of slots at a time: every
            // write lands at or before a slot already read), so the selection
            // passes read only them
            __shared__ int ctot;
            int64_t base = 0;
            for (int64_t c0 = 0; c0 < S; c0 += THREADS) {
                const int64_t t = c0 + tid;
                const int32_t kk = t < S ? key[t] : -1;
                const uint32_t cc = t < S ? cnt[t] : 0u;
                const int pos = block_exclusive_scan<int, THREADS>(kk >= 0 ? 1 : 0, &ctot);
                if (kk >= 0) {
                    key[base + pos] = kk;
                    cnt[base + pos] = cc;
                }
                base += ctot;
            }
            live = base;
            __syncthreads();
        }
        unsigned long long U, W, kth;
        count_and_select<THREADS>(key, cnt, live, jb, topk, sm, U, W, kth);
        if (U == 0) continue;
        // emit the kept entries, both directions
        for (int64_t t = tid; t < live; t += THREADS) {
            const int32_t j = key[t];
            if (j < 0) continue;
            const uint32_t w = cnt[t];
            if ((((W - w) << jb) | (unsigned long long)j) <= kth) emit_edge(i, j, w, jb, ecount, ekey, ew);
        }
    }
}

// exclusive scan of n int64 counts into out[0..n], out[n] = total (copied to the host when asked)
int scan_counts(const int64_t *in, int64_t *out, int64_t n, cudaStream_t s, int64_t *total_host) {
    DBuf<int64_t> tmp;
    SPMM_TRY(tmp.alloc(scan_temp_elems(n), s));
    SPMM_TRY(exclusive_scan<int64_t>(in, out, n, tmp.p, out + n, s));
    if (total_host) SPMM_TRY(to_host(total_host, out + n, 1, s));
    return SPMM_OK;
}

// Stable radix sort of 64-bit keys by their low `bits` (a byte payload rides along).
int sort_keys(DBuf<uint64_t> &k0, DBuf<uint64_t> &k1, int64_t n, int bits, cudaStream_t s) {
    DBuf<uint8_t> v0, v1;
    DBuf<uint32_t> tmp;
    SPMM_TRY(v0.alloc(n, s));
    SPMM_TRY(v1.alloc(n, s));
    SPMM_TRY(tmp.alloc(radix_temp_elems(n), s));
    bool first = true;
    SPMM_TRY(radix_sort_pairs<uint64_t, uint8_t>(k0.p, v0.p, k1.p, v1.p, n, bits, tmp.p, &first, s));
    if (!first) std::swap(k0.p, k1.p);
    return SPMM_OK;
}

// One level's similarity graph as CSR over the n rows (gptr, gcol, gw).
int similarity_graph(const int64_t *ptr, const int32_t *idx, int64_t n, int64_t m, int64_t nnz, uint32_t hub,
                     int64_t topk, DBuf<unsigned long long> &gptr, DBuf<int32_t> &gcol, DBuf<uint32_t> &gw,
                     int64_t *gnnz, cudaStream_t s) {
    *gnnz = 0;
    const int jb = bit_width_u64((uint64_t)(n > 1 ? n - 1 : 1));
    DBuf<uint32_t> deg;
    SPMM_TRY(deg.alloc(m, s));
    SPMM_CUDA_TRY(cudaMemsetAsync(deg.p, 0, (size_t)m * 4, s));
    if (nnz) {
        col_deg_kernel<<<grid_for(nnz, kHemThreads), kHemThreads, 0, s>>>(idx, nnz, deg.p);
        SPMM_LAUNCH_CHECK();
    }
    // pruned pattern (kept columns, in order) and each row's incidence count
    DBuf<int64_t> pcnt, pinc, pptr, pstart;
    SPMM_TRY(pcnt.alloc(n + 1, s));
    SPMM_TRY(pinc.alloc(n + 1, s));
    SPMM_TRY(pptr.alloc(n + 1, s));
    SPMM_TRY(pstart.alloc(n + 1, s));
    prune_kernel<<<warps_grid(n), kHemThreads, 0, s>>>(ptr, idx, n, deg.p, hub, pcnt.p, pinc.p, nullptr, nullptr);
    SPMM_LAUNCH_CHECK();
    int64_t pnnz = 0, npairs = 0;
    SPMM_TRY(scan_counts(pcnt.p, pptr.p, n, s, &pnnz));
    SPMM_TRY(scan_counts(pinc.p, pstart.p, n, s, &npairs));
    if (pnnz == 0 || npairs == 0) return SPMM_OK;
    DBuf<int32_t> pidx;
    SPMM_TRY(pidx.alloc(pnnz, s));
    prune_kernel<<<warps_grid(n), kHemThreads, 0, s>>>(ptr, idx, n, deg.p, hub, nullptr, nullptr, pptr.p, pidx.p);
    SPMM_LAUNCH_CHECK();
    // rows of each kept column
    DBuf<int64_t> tdeg, tptr;
    DBuf<int32_t> trow;
    SPMM_TRY(tdeg.alloc(m + 1, s));
    SPMM_TRY(tptr.alloc(m + 1, s));
    SPMM_TRY(trow.alloc(pnnz, s));
    {
        DBuf<uint32_t> tcur;
        SPMM_TRY(tcur.alloc(m, s));
        SPMM_CUDA_TRY(cudaMemsetAsync(tcur.p, 0, (size_t)m * 4, s));
        col_deg_kernel<<<grid_for(pnnz, kHemThreads), kHemThreads, 0, s>>>(pidx.p, pnnz, tcur.p);
        SPMM_LAUNCH_CHECK();
        widen_kernel<<<grid_for(m, kHemThreads), kHemThreads, 0, s>>>(tcur.p, tdeg.p, m);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(scan_counts(tdeg.p, tptr.p, m, s, nullptr));
        SPMM_CUDA_TRY(cudaMemsetAsync(tcur.p, 0, (size_t)m * 4, s));
        transpose_kernel<<<warps_grid(n), kHemThreads, 0, s>>>(pptr.p, pidx.p, n, tptr.p, tcur.p, trow.p);
        SPMM_LAUNCH_CHECK();
    }
    if (topk == 0) return SPMM_OK;   // no row keeps an edge
    // topk > 0: every row is counted by hashing (hash_topk_kernel); topk < 0
    // (every pair kept): by sorting the rows' incidences in chunks.
    std::vector<int64_t> hstart((size_t)n + 1);
    SPMM_TRY(to_host(hstart.data(), pstart.p, n + 1, s));
    std::vector<int64_t> big;   // rows counted by sorting, ascending
    if (topk < 0)
        for (int64_t r = 0; r < n; ++r)
            if (hstart[r + 1] > hstart[r]) big.push_back(r);
    std::vector<int64_t> bstart(1, 0);
    for (int64_t r : big) bstart.push_back(bstart.back() + hstart[r + 1] - hstart[r]);
    std::vector<std::pair<int64_t, int64_t>> chunks;   // ranges of `big` of at most kPairBudget incidences
    for (size_t b0 = 0; b0 < big.size();) {
        size_t b1 = b0 + 1;
        while (b1 < big.size() && bstart[b1 + 1] - bstart[b0] <= kPairBudget) ++b1;
        chunks.push_back({(int64_t)b0, (int64_t)b1});
        b0 = b1;
    }
    int64_t ecap = 0;
    if (topk > 0) {
        ecap = 2 * n * topk;
    } else {
        for (auto &c : chunks) ecap += 2 * (bstart[c.second] - bstart[c.first]);
    }
    DBuf<uint64_t> ek0, ek1;
    DBuf<uint32_t> ew0;
    SPMM_TRY(ek0.alloc(ecap, s));
    SPMM_TRY(ew0.alloc(ecap, s));
    int64_t ecount = 0;
    DBuf<int64_t> dlist, dstart;
    if (topk > 0) {
        // global tables for the rows whose table exceeds shared memory
        std::vector<int64_t> hoff((size_t)n + 1, 0);
        int64_t gslots = 0;
        for (int64_t r = 0; r < n; ++r) {
            hoff[r] = gslots;
            const int64_t S = table_slots(hstart[r + 1] - hstart[r]);
            if (S > kMidSlots) gslots += S;
        }
        DBuf<int64_t> goff;
        DBuf<int32_t> gkey;
        DBuf<uint32_t> gcnt;
        SPMM_TRY(goff.alloc(n + 1, s));
        SPMM_CUDA_TRY(cudaMemcpyAsync(goff.p, hoff.data(), (size_t)(n + 1) * 8, cudaMemcpyHostToDevice, s));
        SPMM_TRY(gkey.alloc(gslots, s));
        SPMM_TRY(gcnt.alloc(gslots, s));
        DBuf<unsigned long long> ecnt;
        SPMM_TRY(ecnt.alloc(1, s));
        SPMM_CUDA_TRY(cudaMemsetAsync(ecnt.p, 0, 8, s));
        auto tiny = hash_topk_kernel<kHashThreads, kTinySlots>;
        auto small = hash_topk_kernel<kHashThreads, kSmemSlots>;
        auto mid = hash_topk_kernel<512, kMidSlots>;
        SPMM_CUDA_TRY(cudaFuncSetAttribute(tiny, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)((size_t)kTinySlots * 8)));
        SPMM_CUDA_TRY(cudaFuncSetAttribute(small, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)((size_t)kSmemSlots * 8)));
        SPMM_CUDA_TRY(cudaFuncSetAttribute(mid, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)((size_t)kMidSlots * 8)));
        int dev = 0, sms = 0, per_sm = 0;
        SPMM_CUDA_TRY(cudaGetDevice(&dev));
        SPMM_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        SPMM_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tiny, kHashThreads,
                                                                    (size_t)kTinySlots * 8));
        tiny<<<(unsigned)std::min<int64_t>(n, (int64_t)sms * std::max(per_sm, 1)), kHashThreads,
               (size_t)kTinySlots * 8, s>>>(pptr.p, pidx.p, tptr.p, trow.p, pinc.p, goff.p, gkey.p, gcnt.p, n, jb,
                                            topk, ecnt.p, ek0.p, ew0.p);
        SPMM_LAUNCH_CHECK();
        const int64_t grid = std::min<int64_t>(n, (int64_t)sms * 3);
        small<<<(unsigned)grid, kHashThreads, (size_t)kSmemSlots * 8, s>>>(
            pptr.p, pidx.p, tptr.p, trow.p, pinc.p, goff.p, gkey.p, gcnt.p, n, jb, topk, ecnt.p, ek0.p, ew0.p);
        SPMM_LAUNCH_CHECK();
        mid<<<(unsigned)std::min<int64_t>(n, sms), 512, (size_t)kMidSlots * 8, s>>>(
            pptr.p, pidx.p, tptr.p, trow.p, pinc.p, goff.p, gkey.p, gcnt.p, n, jb, topk, ecnt.p, ek0.p, ew0.p);
        SPMM_LAUNCH_CHECK();
        if (gslots > 0) {   // rows with global tables: 1,024 threads each
            hash_topk_kernel<1024, 0><<<(unsigned)std::min<int64_t>(n, sms * 2), 1024, 0, s>>>(
                pptr.p, pidx.p, tptr.p, trow.p, pinc.p, goff.p, gkey.p, gcnt.p, n, jb, topk, ecnt.p, ek0.p, ew0.p);
            SPMM_LAUNCH_CHECK();
        }
        unsigned long long ec = 0;
        SPMM_TRY(to_host(&ec, ecnt.p, 1, s));
        ecount = (int64_t)ec;
    }
    if (!big.empty()) {
        // heaviest possible w: the longest pruned row among them
        int64_t wmax_len = 0;
        {
            std::vector<int64_t> hp((size_t)n + 1);
            SPMM_TRY(to_host(hp.data(), pptr.p, n + 1, s));
            for (int64_t r : big) wmax_len = std::max(wmax_len, hp[r + 1] - hp[r]);
        }
        const int wb = bit_width_u64((uint64_t)wmax_len + 1);
        SPMM_TRY(dlist.alloc((int64_t)big.size(), s));
        SPMM_TRY(dstart.alloc((int64_t)bstart.size(), s));
        SPMM_CUDA_TRY(cudaMemcpyAsync(dlist.p, big.data(), big.size() * 8, cudaMemcpyHostToDevice, s));
        SPMM_CUDA_TRY(cudaMemcpyAsync(dstart.p, bstart.data(), bstart.size() * 8, cudaMemcpyHostToDevice, s));
        for (auto &c : chunks) {
            const int64_t b0 = c.first, rows = c.second - c.first;
            const int64_t P = bstart[c.second] - bstart[b0];
            if (P == 0) continue;
            const int rb = bit_width_u64((uint64_t)rows);
            if (rb + jb > 63 || rb + wb + jb > 64) return SPMM_EUNSUPPORTED;
            const uint64_t sentinel = (rb + jb == 64) ? ~0ull : ((1ull << (rb + jb)) - 1ull);
            DBuf<uint64_t> k0, k1;
            SPMM_TRY(k0.alloc(P, s));
            SPMM_TRY(k1.alloc(P, s));
            gen_pairs_kernel<<<warps_grid(rows), kHemThreads, 0, s>>>(pptr.p, pidx.p, tptr.p, trow.p, dlist.p + b0,
                                                                      dstart.p + b0, rows, jb, sentinel, k0.p);
            SPMM_LAUNCH_CHECK();
            SPMM_TRY(sort_keys(k0, k1, P, rb + jb, s));
            // unique pairs with their counts, keyed for the top-k order
            DBuf<int64_t> flag, pos;
            SPMM_TRY(flag.alloc(P + 1, s));
            SPMM_TRY(pos.alloc(P + 1, s));
            head_flags_kernel<<<grid_for(P, kHemThreads), kHemThreads, 0, s>>>(k0.p, P, sentinel, flag.p);
            SPMM_LAUNCH_CHECK();
            int64_t U = 0;
            SPMM_TRY(scan_counts(flag.p, pos.p, P, s, &U));
            if (U == 0) continue;
            DBuf<uint64_t> u0, u1;
            SPMM_TRY(u0.alloc(U, s));
            SPMM_TRY(u1.alloc(U, s));
            rle_kernel<<<grid_for(P, kHemThreads), kHemThreads, 0, s>>>(k0.p, P, sentinel, pos.p, jb, wb, u0.p);
            SPMM_LAUNCH_CHECK();
            k0.release();
            k1.release();
            SPMM_TRY(sort_keys(u0, u1, U, rb + wb + jb, s));
            topk_flags_kernel<<<grid_for(U, kHemThreads), kHemThreads, 0, s>>>(u0.p, U, jb, wb, topk, flag.p);
            SPMM_LAUNCH_CHECK();
            int64_t kept = 0;
            SPMM_TRY(scan_counts(flag.p, pos.p, U, s, &kept));
            if (ecount + 2 * kept > ecap) return SPMM_EUNSUPPORTED;
            topk_emit_kernel<<<grid_for(U, kHemThreads), kHemThreads, 0, s>>>(u0.p, U, flag.p, pos.p, dlist.p + b0,
                                                                              jb, wb, ecount, ek0.p, ew0.p);
            SPMM_LAUNCH_CHECK();
            ecount += 2 * kept;
        }
    }
    pidx.release();
    trow.release();
    if (ecount == 0) return SPMM_OK;
    // symmetric graph: sort (row, col) keys with their weights, drop repeats
    DBuf<uint32_t> ew1;
    DBuf<uint32_t> tmp;
    SPMM_TRY(ek1.alloc(ecount, s));
    SPMM_TRY(ew1.alloc(ecount, s));
    SPMM_TRY(tmp.alloc(radix_temp_elems(ecount), s));
    bool first = true;
    SPMM_TRY(radix_sort_pairs<uint64_t, uint32_t>(ek0.p, ew0.p, ek1.p, ew1.p, ecount, 2 * jb, tmp.p, &first, s));
    const uint64_t *ek = first ? ek0.p : ek1.p;
    const uint32_t *ew = first ? ew0.p : ew1.p;
    DBuf<int64_t> flag, pos;
    SPMM_TRY(flag.alloc(ecount + 1, s));
    SPMM_TRY(pos.alloc(ecount + 1, s));
    DBuf<unsigned long long> rowcnt;
    SPMM_TRY(rowcnt.alloc(n + 1, s));
    SPMM_CUDA_TRY(cudaMemsetAsync(rowcnt.p, 0, (size_t)(n + 1) * 8, s));
    edge_heads_kernel<<<grid_for(ecount, kHemThreads), kHemThreads, 0, s>>>(ek, ecount, flag.p, jb, rowcnt.p);
    SPMM_LAUNCH_CHECK();
    int64_t G = 0;
    SPMM_TRY(scan_counts(flag.p, pos.p, ecount, s, &G));
    SPMM_TRY(gptr.alloc(n + 1, s));
    SPMM_TRY(gcol.alloc(G, s));
    SPMM_TRY(gw.alloc(G, s));
    {
        DBuf<unsigned long long> tmp2;
        SPMM_TRY(tmp2.alloc(scan_temp_elems(n + 1), s));
        SPMM_TRY(exclusive_scan<unsigned long long>(rowcnt.p, gptr.p, n + 1, tmp2.p, nullptr, s));
    }
    edge_emit_kernel<<<grid_for(ecount, kHemThreads), kHemThreads, 0, s>>>(ek, ew, ecount, flag.p, pos.p, jb,
                                                                           gcol.p, gw.p);
    SPMM_LAUNCH_CHECK();
    *gnnz = G;
    return SPMM_OK;
}

}  // namespace
}  // namespace spmm

using namespace spmm;

// Levels the matching loop may run for `target` (the reference's cap,
// clustering.py:291-296): 8 * max(1, ceil(log2(target))) + 16.
// Keeps the device's default stream-ordered pool from returning its memory to
// the system at every synchronisation while the levels run (each level frees
// and re-allocates gigabytes of scratch; remapping it cost more than the
// kernels).  When the call ends the pool is trimmed to its previous release
// threshold and that threshold is restored.
class PoolHold {
  public:
    explicit PoolHold(cudaStream_t s) : s_(s) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetDefaultMemPool(&pool_, dev) != cudaSuccess) return;
        if (cudaMemPoolGetAttribute(pool_, cudaMemPoolAttrReleaseThreshold, &old_) != cudaSuccess) return;
        uint64_t keep = ~0ull;
        held_ = cudaMemPoolSetAttribute(pool_, cudaMemPoolAttrReleaseThreshold, &keep) == cudaSuccess;
    }
    PoolHold(const PoolHold &) = delete;
    PoolHold &operator=(const PoolHold &) = delete;
    ~PoolHold() {
        if (!held_) return;
        cudaStreamSynchronize(s_);                  // the levels' frees have completed
        cudaMemPoolTrimTo(pool_, (size_t)old_);
        cudaMemPoolSetAttribute(pool_, cudaMemPoolAttrReleaseThreshold, &old_);
    }

  private:
    cudaStream_t s_;
    cudaMemPool_t pool_{};
    uint64_t old_ = 0;
    bool held_ = false;
};

static int hem_max_levels(int64_t target) {
    int lg = 0;
    while ((1ll << lg) < target) ++lg;
    return 8 * (lg > 1 ? lg : 1) + 16;
}

extern "C" int64_t spmm_hem_level_slots(int64_t target) { return (int64_t)hem_max_levels(target) + 1; }

extern "C" int spmm_hem_hierarchy(int64_t rows, int64_t cols, const int64_t *indptr, const int32_t *indices,
                                  int64_t target, int64_t max_size, int64_t max_nnz, int64_t hub_degree, int64_t topk,
                                  int32_t residual_rounds, int32_t feasible_first, int64_t *labels, int64_t *levels,
                                  int64_t level_slots, int64_t *n_levels, spmm_stream_t stream) {
    if (rows < 0 || cols < 0 || !labels || (rows > 0 && !indptr) || hub_degree < 0 || residual_rounds < 0)
        return SPMM_EINVAL;
    if (levels && (!n_levels || level_slots < spmm_hem_level_slots(target))) return SPMM_EINVAL;
    if (rows > 0x7fffffffLL || cols > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    cudaStream_t s = (cudaStream_t)stream;
    int64_t recorded = 0;
    if (n_levels) *n_levels = 0;
    if (rows == 0) return SPMM_OK;
    iota64_kernel<<<grid_for(rows, kHemThreads), kHemThreads, 0, s>>>(labels, rows);
    SPMM_LAUNCH_CHECK();
    // levels[k][rows]: identity, then the labels after each level that matched
    auto record = [&]() -> int {
        if (!levels) return SPMM_OK;
        SPMM_CUDA_TRY(cudaMemcpyAsync(levels + recorded * rows, labels, (size_t)rows * 8, cudaMemcpyDeviceToDevice, s));
        *n_levels = ++recorded;
        return SPMM_OK;
    };
    SPMM_TRY(record());
    if (rows <= 1 || target <= 1) return levels ? (cudaStreamSynchronize(s) == cudaSuccess ? SPMM_OK : SPMM_ECUDA)
                                                : SPMM_OK;
    const PoolHold hold(s);   // declared before every level buffer: released after them
    int64_t nnz0 = 0;
    SPMM_TRY(to_host(&nnz0, indptr + rows, 1, s));
    const Caps caps{max_size, max_nnz};
    // level state: pattern (ptr, idx) of n rows, sizes and nnz of its rows
    int64_t n = rows, nnz = nnz0;
    DBuf<int64_t> lptr, size, rnnz;
    DBuf<int32_t> lidx;
    SPMM_TRY(lptr.alloc(n + 1, s));
    SPMM_TRY(lidx.alloc(nnz, s));
    SPMM_CUDA_TRY(cudaMemcpyAsync(lptr.p, indptr, (size_t)(n + 1) * 8, cudaMemcpyDeviceToDevice, s));
    if (nnz) SPMM_CUDA_TRY(cudaMemcpyAsync(lidx.p, indices, (size_t)nnz * 4, cudaMemcpyDeviceToDevice, s));
    SPMM_TRY(size.alloc(n, s));
    SPMM_TRY(rnnz.alloc(n, s));
    fill_kernel<<<grid_for(n, kHemThreads), kHemThreads, 0, s>>>(size.p, n, 1);
    SPMM_LAUNCH_CHECK();
    diff_kernel<<<grid_for(n, kHemThreads), kHemThreads, 0, s>>>(lptr.p, n, rnnz.p);
    SPMM_LAUNCH_CHECK();
    const int max_levels = hem_max_levels(target);
    DBuf<unsigned long long> matched;
    SPMM_TRY(matched.alloc(1, s));
    for (int level = 0; level < max_levels && n > 1; ++level) {
        DBuf<unsigned long long> gptr;
        DBuf<int32_t> gcol;
        DBuf<uint32_t> gw;
        int64_t gnnz = 0;
        SPMM_TRY(similarity_graph(lptr.p, lidx.p, n, cols, nnz, (uint32_t)std::min<int64_t>(hub_degree, 0xFFFFFFFFll),
                                  topk, gptr, gcol, gw, &gnnz, s));
        if (gnnz == 0) break;
        DBuf<uint8_t> active;
        DBuf<int64_t> best, mate;
        SPMM_TRY(active.alloc(n, s));
        SPMM_TRY(best.alloc(n, s));
        SPMM_TRY(mate.alloc(n, s));
        SPMM_CUDA_TRY(cudaMemsetAsync(active.p, 1, (size_t)n, s));
        fill_kernel<<<grid_for(n, kHemThreads), kHemThreads, 0, s>>>(mate.p, n, -1);
        SPMM_LAUNCH_CHECK();
        // vertices with many edges, picked by a CTA each
        DBuf<int64_t> heavy;
        SPMM_TRY(heavy.alloc(n, s));
        SPMM_CUDA_TRY(cudaMemsetAsync(matched.p, 0, 8, s));
        heavy_list_kernel<<<grid_for(n, kHemThreads), kHemThreads, 0, s>>>(gptr.p, n, matched.p, heavy.p);
        SPMM_LAUNCH_CHECK();
        unsigned long long n_heavy = 0;
        SPMM_TRY(to_host(&n_heavy, matched.p, 1, s));
        unsigned long long total = 0;
        for (int round = 0; round < residual_rounds; ++round) {
            SPMM_CUDA_TRY(cudaMemsetAsync(matched.p, 0, 8, s));
            best_kernel<<<warps_grid(n), kHemThreads, 0, s>>>(gptr.p, gcol.p, gw.p, n, active.p, size.p, rnnz.p,
                                                               caps, feasible_first, best.p);
            SPMM_LAUNCH_CHECK();
            if (n_heavy) {
                best_heavy_kernel<<<(unsigned)std::min<unsigned long long>(n_heavy, 148ull * 8), kHeavyThreads, 0,
                                    s>>>(gptr.p, gcol.p, gw.p, heavy.p, (int64_t)n_heavy, active.p, size.p, rnnz.p,
                                         caps, feasible_first, best.p);
                SPMM_LAUNCH_CHECK();
            }
            mutual_kernel<<<grid_for(n, kHemThreads), kHemThreads, 0, s>>>(best.p, n, size.p, rnnz.p, caps, mate.p,
                                                                          active.p, matched.p);
            SPMM_LAUNCH_CHECK();
            unsigned long long got = 0;
            SPMM_TRY(to_host(&got, matched.p, 1, s));
            if (got == 0) break;
            total += got;
        }
        if (total == 0) break;
        // contraction
        DBuf<int64_t> flag, rank, new_id, nlen, nptr;
        SPMM_TRY(flag.alloc(n + 1, s));
        SPMM_TRY(rank.alloc(n + 1, s));
        root_flags_kernel<<<grid_for(n, kHemThreads), kHemThreads, 0, s>>>(mate.p, n, flag.p);
        SPMM_LAUNCH_CHECK();
        int64_t n_new = 0;
        SPMM_TRY(scan_counts(flag.p, rank.p, n, s, &n_new));
        DBuf<unsigned long long> nsize, nnnz;
        SPMM_TRY(new_id.alloc(n, s));
        SPMM_TRY(nlen.alloc(n_new + 1, s));
        SPMM_TRY(nptr.alloc(n_new + 1, s));
        SPMM_TRY(nsize.alloc(n_new, s));
        SPMM_TRY(nnnz.alloc(n_new, s));
        SPMM_CUDA_TRY(cudaMemsetAsync(nsize.p, 0, (size_t)n_new * 8, s));
        SPMM_CUDA_TRY(cudaMemsetAsync(nnnz.p, 0, (size_t)n_new * 8, s));
        contract_kernel<<<warps_grid(n), kHemThreads, 0, s>>>(mate.p, n, rank.p, size.p, rnnz.p, lptr.p,
                                                                        lidx.p, new_id.p, nsize.p, nnnz.p, nlen.p);
        SPMM_LAUNCH_CHECK();
        int64_t nnz_new = 0;
        SPMM_TRY(scan_counts(nlen.p, nptr.p, n_new, s, &nnz_new));
        DBuf<int32_t> nidx;
        SPMM_TRY(nidx.alloc(nnz_new, s));
        contract_emit_kernel<<<warps_grid(n), kHemThreads, 0, s>>>(mate.p, n, rank.p, lptr.p, lidx.p,
                                                                             nptr.p, nidx.p);
        SPMM_LAUNCH_CHECK();
        relabel_kernel<<<grid_for(rows, kHemThreads), kHemThreads, 0, s>>>(labels, rows, new_id.p);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(record());
        SPMM_TRY(size.alloc(n_new, s));
        SPMM_TRY(rnnz.alloc(n_new, s));
        copy_cast_kernel<int64_t><<<grid_for(n_new, kHemThreads), kHemThreads, 0, s>>>(nsize.p, size.p, n_new);
        SPMM_LAUNCH_CHECK();
        copy_cast_kernel<int64_t><<<grid_for(n_new, kHemThreads), kHemThreads, 0, s>>>(nnnz.p, rnnz.p, n_new);
        SPMM_LAUNCH_CHECK();
        std::swap(lptr.p, nptr.p);
        std::swap(lidx.p, nidx.p);
        n = n_new;
        nnz = nnz_new;
    }
    SPMM_CUDA_TRY(cudaStreamSynchronize(s));
    return SPMM_OK;
}

extern "C" int spmm_hem_labels(int64_t rows, int64_t cols, const int64_t *indptr, const int32_t *indices,
                               int64_t target, int64_t max_size, int64_t max_nnz, int64_t hub_degree, int64_t topk,
                               int32_t residual_rounds, int32_t feasible_first, int64_t *labels,
                               spmm_stream_t stream) {
    return spmm_hem_hierarchy(rows, cols, indptr, indices, target, max_size, max_nnz, hub_degree, topk,
                              residual_rounds, feasible_first, labels, nullptr, 0, nullptr, stream);
}
