// spmm_common.cuh -- vector load/store and accumulation helpers of the SpMM
// kernels.
#pragma once

#include "common.cuh"

namespace spmm {

// First index i in [0, n) with a[i] >= key (a ascending), by a 32-way search
// of the whole warp.
__device__ __forceinline__ int64_t warp_lower_bound(const int32_t *a, int64_t n, int64_t key, int lane) {
    int64_t lo = 0, hi = n;
    while (hi - lo > 32) {
        const int64_t step = (hi - lo + 31) / 32;
        const int64_t pi = lo + lane * step;
        const bool pred = pi < hi && (int64_t)__ldg(a + pi) < key;
        const int c = __popc(__ballot_sync(kFullMask, pred));
        if (c == 0) return lo;
        const int64_t nhi = lo + c * step;
        lo = lo + (c - 1) * step + 1;
        hi = nhi < hi ? nhi : hi;
    }
    const int64_t pi = lo + lane;
    const bool pred = pi < hi && (int64_t)__ldg(a + pi) < key;
    return lo + __popc(__ballot_sync(kFullMask, pred));
}

// One past the last block of row group rg, scanning forward from b (the
// first block with row group >= rg); row groups hold a handful of blocks.
__device__ __forceinline__ int64_t group_end(const int32_t *blk_row_grp, int64_t nb, int64_t b, int64_t rg,
                                             int lane) {
    for (;; b += 32) {
        const int64_t i = b + lane;
        const bool in = i < nb && (int64_t)__ldg(blk_row_grp + i) <= rg;
        const unsigned m = __ballot_sync(kFullMask, in);
        if (m != kFullMask) return b + __popc(m);   // the group's blocks are a prefix
    }
}

// VEC consecutive scalars moved as one 4/8/16-byte access.
template <typename S, int VEC> struct VecOf;
template <> struct VecOf<float, 1> { using T = float; };
template <> struct VecOf<float, 2> { using T = float2; };
template <> struct VecOf<float, 4> { using T = float4; };
template <> struct VecOf<double, 1> { using T = double; };
template <> struct VecOf<double, 2> { using T = double2; };

template <typename S, int VEC>
struct Frag {
    S v[VEC];
};

template <typename S, int VEC>
__device__ __forceinline__ Frag<S, VEC> ldg_frag(const S *p) {
    using V = typename VecOf<S, VEC>::T;
    V t = __ldg(reinterpret_cast<const V *>(p));
    Frag<S, VEC> f;
    static_assert(sizeof(V) == sizeof(f), "vector size");
    memcpy(&f, &t, sizeof(V));
    return f;
}

// From shared memory, as one vector access.
template <typename S, int VEC>
__device__ __forceinline__ Frag<S, VEC> lds_frag(const S *p) {
    using V = typename VecOf<S, VEC>::T;
    const V t = *reinterpret_cast<const V *>(p);
    Frag<S, VEC> f;
    memcpy(&f, &t, sizeof(V));
    return f;
}

template <typename S, int VEC>
__device__ __forceinline__ void st_frag(S *p, const Frag<S, VEC> &f) {
    using V = typename VecOf<S, VEC>::T;
    V t;
    memcpy(&t, &f, sizeof(V));
    __stcs(reinterpret_cast<V *>(p), t);  // Y is written once: streaming store
}

// acc[v] += a * X[col][feature slot v] for VPT slots of VEC scalars; slot v of
// lane l covers features base + (v * LPR + l) * VEC.
template <typename S, int VEC, int VPT, int LPR>
struct RowAcc {
    Frag<S, VEC> a[VPT];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int v = 0; v < VPT; ++v)
#pragma unroll
            for (int e = 0; e < VEC; ++e) a[v].v[e] = S(0);
    }
};

}  // namespace spmm
