// common.cuh -- shared helpers of the spmm_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/spmm_b200.h"

namespace spmm {

constexpr unsigned kFullMask = 0xffffffffu;

// Status plumbing: every host routine returns an spmm_status; CUDA failures
// are mapped to SPMM_ECUDA and never thrown.
#define SPMM_CUDA_TRY(...)                        \
    do {                                          \
        cudaError_t _e = (__VA_ARGS__);           \
        if (_e != cudaSuccess) return SPMM_ECUDA; \
    } while (0)

#define SPMM_LAUNCH_CHECK()                                   \
    do {                                                      \
        if (cudaPeekAtLastError() != cudaSuccess) {           \
            (void)cudaGetLastError();                         \
            return SPMM_ECUDA;                                \
        }                                                     \
    } while (0)

// Host-side count of product-kernel launches (spmm_product_launches).
void note_product_launch();

// SPMM_LAUNCH_CHECK for a product kernel: also counts the launch.
#define SPMM_PRODUCT_LAUNCHED()      \
    do {                             \
        SPMM_LAUNCH_CHECK();         \
        ::spmm::note_product_launch(); \
    } while (0)

#define SPMM_TRY(...)              \
    do {                           \
        int _s = (__VA_ARGS__);    \
        if (_s != SPMM_OK) return _s; \
    } while (0)

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of bits needed to represent v (0 -> 0).
inline int bit_width_u64(uint64_t v) {
    int b = 0;
    while (v) { ++b; v >>= 1; }
    return b;
}

// Grid size for grid-stride loops: a few waves of 148 SMs, capped by the work.
inline unsigned grid_for(int64_t n, int threads) {
    int64_t blocks = ceil_div(n, threads);
    const int64_t cap = 148LL * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

// Bump allocator over a caller-owned workspace.  Every carve is 256-B aligned
// so vector and bulk accesses stay aligned.
struct Arena {
    char *base;
    size_t cap;
    size_t used;
    __host__ explicit Arena(void *p, size_t c) : base((char *)p), cap(c), used(0) {}
    template <typename T>
    __host__ T *take(int64_t n) {
        size_t bytes = (size_t)(n > 0 ? n : 1) * sizeof(T);
        size_t off = (used + 255) & ~(size_t)255;
        used = off + bytes;
        if (base == nullptr || used > cap) return nullptr;
        return (T *)(base + off);
    }
};

// Size-only pass of the same carve sequence (base == nullptr).
template <typename T>
inline void arena_count(size_t &used, int64_t n) {
    size_t bytes = (size_t)(n > 0 ? n : 1) * sizeof(T);
    used = ((used + 255) & ~(size_t)255) + bytes;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// ---------------------------------------------------------------------------
// Exclusive scan (three kernels: per-tile reduce, single-CTA scan of the tile
// sums, per-tile scan + offset).  T is an unsigned or signed integer type.
// ---------------------------------------------------------------------------
constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T n = __shfl_up_sync(kFullMask, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total to *total.
template <typename T, int THREADS>
__device__ __forceinline__ T block_exclusive_scan(T v, T *total) {
    __shared__ T warp_sums[THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T inc = warp_inclusive_scan(v);
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        T s = lane < THREADS / 32 ? warp_sums[lane] : T(0);
        T si = warp_inclusive_scan(s);
        if (lane < THREADS / 32) warp_sums[lane] = si - s;
        if (lane == THREADS / 32 - 1) *total = si;
    }
    __syncthreads();
    T res = inc - v + warp_sums[warp];
    __syncthreads();
    return res;
}

template <typename T>
__global__ void scan_reduce_kernel(const T *__restrict__ in, int64_t n, T *__restrict__ sums) {
    const int64_t base = (int64_t)blockIdx.x * kScanTile;
    T s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        int64_t k = base + (int64_t)i * kScanThreads + threadIdx.x;
        if (k < n) s += in[k];
    }
    __shared__ T tot;
    block_exclusive_scan<T, kScanThreads>(s, &tot);
    if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

// One CTA scans `n` tile sums in place (exclusive); writes the grand total.
template <typename T>
__global__ void scan_sums_kernel(T *__restrict__ sums, int64_t n, T *__restrict__ total) {
    __shared__ T carry;
    __shared__ T tot;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int64_t base = 0; base < n; base += kScanThreads) {
        int64_t k = base + threadIdx.x;
        T v = k < n ? sums[k] : T(0);
        T ex = block_exclusive_scan<T, kScanThreads>(v, &tot);
        if (k < n) sums[k] = ex + carry;
        __syncthreads();
        if (threadIdx.x == 0) carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0 && total) *total = carry;
}

template <typename T>
__global__ void scan_apply_kernel(const T *__restrict__ in, T *__restrict__ out, int64_t n,
                                  const T *__restrict__ offsets) {
    // Blocked arrangement inside the tile: thread t owns items [t*8, t*8+8).
    const int64_t base = (int64_t)blockIdx.x * kScanTile + (int64_t)threadIdx.x * kScanItems;
    T v[kScanItems];
    T s = 0;
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        v[i] = (base + i < n) ? in[base + i] : T(0);
        s += v[i];
    }
    __shared__ T tot;
    T run = block_exclusive_scan<T, kScanThreads>(s, &tot) + offsets[blockIdx.x];
#pragma unroll
    for (int i = 0; i < kScanItems; ++i) {
        if (base + i < n) out[base + i] = run;
        run += v[i];
    }
}

// Workspace (elements of T) needed by exclusive_scan for n items.
inline int64_t scan_temp_elems(int64_t n) { return ceil_div(n > 0 ? n : 1, kScanTile) + 1; }

// out[i] = sum(in[0..i)), total (device pointer, may be null) = sum(in).
// `in` and `out` may alias.  temp needs scan_temp_elems(n) elements.
template <typename T>
int exclusive_scan(const T *in, T *out, int64_t n, T *temp, T *total, cudaStream_t s) {
    if (n <= 0) {
        if (total) SPMM_CUDA_TRY(cudaMemsetAsync(total, 0, sizeof(T), s));
        return SPMM_OK;
    }
    int64_t tiles = ceil_div(n, kScanTile);
    if (tiles > 0x7fffffffLL) return SPMM_EUNSUPPORTED;
    scan_reduce_kernel<T><<<(unsigned)tiles, kScanThreads, 0, s>>>(in, n, temp);
    SPMM_LAUNCH_CHECK();
    scan_sums_kernel<T><<<1, kScanThreads, 0, s>>>(temp, tiles, total);
    SPMM_LAUNCH_CHECK();
    scan_apply_kernel<T><<<(unsigned)tiles, kScanThreads, 0, s>>>(in, out, n, temp);
    SPMM_LAUNCH_CHECK();
    return SPMM_OK;
}

// ---------------------------------------------------------------------------
// Stable LSD radix sort of (key, value) pairs, 8 bits per pass.
//
// Tile = 256 threads x 8 rounds = 2048 items in a warp-striped arrangement:
// item (warp w, round i, lane l) sits at tile position w*256 + i*32 + l.  Each
// pass: (1) per-tile digit histogram, (2) exclusive scan of the histograms in
// digit-major / tile-minor order, (3) scatter, where an item's rank among
// equal digits of its tile comes from __match_any_sync peers and per-warp
// running counters -- which keeps equal keys in input order (stable).
// ---------------------------------------------------------------------------
constexpr int kSortThreads = 256;
constexpr int kSortRounds = 8;
constexpr int kSortTile = kSortThreads * kSortRounds;
constexpr int kSortWarps = kSortThreads / 32;

template <typename K>
__global__ void radix_hist_kernel(const K *__restrict__ keys, int64_t n, int shift,
                                  uint32_t *__restrict__ hist, int64_t tiles) {
    __shared__ uint32_t h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kSortTile;
#pragma unroll
    for (int i = 0; i < kSortRounds; ++i) {
        int64_t k = base + (int64_t)i * kSortThreads + threadIdx.x;
        if (k < n) atomicAdd(&h[(uint32_t)(keys[k] >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    hist[(int64_t)threadIdx.x * tiles + blockIdx.x] = h[threadIdx.x];
}

template <typename K, typename V>
__global__ void radix_scatter_kernel(const K *__restrict__ kin, const V *__restrict__ vin,
                                     K *__restrict__ kout, V *__restrict__ vout, int64_t n,
                                     int shift, const uint32_t *__restrict__ offsets,
                                     int64_t tiles) {
    __shared__ uint32_t wh[kSortWarps][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int d = threadIdx.x; d < kSortWarps * 256; d += kSortThreads) (&wh[0][0])[d] = 0;
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * kSortTile + (int64_t)warp * 256;
    K key[kSortRounds];
    uint32_t rank[kSortRounds];
    uint32_t dig[kSortRounds];
    const unsigned lt = lanemask_lt();
#pragma unroll
    for (int i = 0; i < kSortRounds; ++i) {
        const int64_t k = base + i * 32 + lane;
        const bool valid = k < n;
        key[i] = valid ? kin[k] : K(0);
        const uint32_t d = valid ? ((uint32_t)(key[i] >> shift) & 0xFF) : 256u;
        dig[i] = d;
        const unsigned peers = __match_any_sync(kFullMask, d);
        uint32_t before = 0;
        if (valid) before = wh[warp][d];
        __syncwarp();
        if (valid && lane == __ffs(peers) - 1) wh[warp][d] = before + __popc(peers);
        __syncwarp();
        rank[i] = before + __popc(peers & lt);
    }
    __syncthreads();
    {
        // exclusive prefix over warps for digit threadIdx.x
        uint32_t run = 0;
#pragma unroll
        for (int w = 0; w < kSortWarps; ++w) {
            uint32_t t = wh[w][threadIdx.x];
            wh[w][threadIdx.x] = run;
            run += t;
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kSortRounds; ++i) {
        const int64_t k = base + i * 32 + lane;
        if (k < n) {
            const uint32_t d = dig[i];
            const uint32_t pos = offsets[(int64_t)d * tiles + blockIdx.x] + wh[warp][d] + rank[i];
            kout[pos] = key[i];
            vout[pos] = vin[k];
        }
    }
}

inline int64_t radix_tiles(int64_t n) { return ceil_div(n > 0 ? n : 1, kSortTile); }
// uint32 elements of temp storage radix_sort_pairs needs.
inline int64_t radix_temp_elems(int64_t n) {
    int64_t h = 256 * radix_tiles(n);
    return h + scan_temp_elems(h);
}

// Sorts n pairs by bits [0, key_bits) of the key, stably.  Data ping-pongs
// between (k0, v0) and (k1, v1); on return *result_in_first says which pair of
// buffers holds the sorted output.
template <typename K, typename V>
int radix_sort_pairs(K *k0, V *v0, K *k1, V *v1, int64_t n, int key_bits, uint32_t *temp,
                     bool *result_in_first, cudaStream_t s) {
    *result_in_first = true;
    if (n <= 1 || key_bits <= 0) return SPMM_OK;
    if (n > 0xFFFFFFFFLL) return SPMM_EUNSUPPORTED;
    const int64_t tiles = radix_tiles(n);
    uint32_t *hist = temp;
    uint32_t *stemp = temp + 256 * tiles;
    bool first = true;
    for (int shift = 0; shift < key_bits; shift += 8) {
        const K *ki = first ? k0 : k1;
        const V *vi = first ? v0 : v1;
        K *ko = first ? k1 : k0;
        V *vo = first ? v1 : v0;
        radix_hist_kernel<K><<<(unsigned)tiles, kSortThreads, 0, s>>>(ki, n, shift, hist, tiles);
        SPMM_LAUNCH_CHECK();
        SPMM_TRY(exclusive_scan<uint32_t>(hist, hist, 256 * tiles, stemp, nullptr, s));
        radix_scatter_kernel<K, V><<<(unsigned)tiles, kSortThreads, 0, s>>>(ki, vi, ko, vo, n, shift,
                                                                            hist, tiles);
        SPMM_LAUNCH_CHECK();
        first = !first;
    }
    *result_in_first = first;
    return SPMM_OK;
}

// out[i] = i for i < n.
template <typename T>
__global__ void iota_kernel(T *__restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (T)i;
}

// Order-preserving unsigned image of a float / double, matching operator< on
// non-NaN values except that -0.0 sorts before +0.0.
__device__ __forceinline__ uint64_t order_key(float v) {
    uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? (uint64_t)(~u) : (uint64_t)(u | 0x80000000u);
}
__device__ __forceinline__ uint64_t order_key(double v) {
    uint64_t u = (uint64_t)__double_as_longlong(v);
    return (u >> 63) ? ~u : (u | (1ULL << 63));
}

}  // namespace spmm
