// spmm_common.cuh -- vector load/store and accumulation helpers of the SpMM
// kernels.
#pragma once

#include "common.cuh"

namespace spmm {

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
