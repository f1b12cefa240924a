// reduce_state.cuh - per-lane reduction state of the reduction kernels
// (reduce.cu) and the fused chain reduction (eltwise.cu): the running value
// and, for arg kinds, its index; element folds, pairwise combine with a fixed
// lane order, and the warp butterfly.
//
// Semantics shared by every path: sums accumulate in the compute type; max /
// min propagate NaN (a NaN sticks once seen); argmax / argmin keep the first
// index of the extreme, a NaN counting as the extreme; a state with no
// element yet has index -1.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace tadma_b200 {
namespace {

enum Kind { K_SUM = 0, K_MAX = 1, K_MIN = 2, K_ARGMAX = 3, K_ARGMIN = 4 };

// A squared element (sum of squares, variance): one rounded multiply, never
// contracted into the fold's add, as a materialised square would be.
__device__ __forceinline__ float sq(float v) { return __fmul_rn(v, v); }
__device__ __forceinline__ double sq(double v) { return __dmul_rn(v, v); }
__device__ __forceinline__ int64_t sq(int64_t v) { return v * v; }

// ------------------------------------------------------------ state ops --

template <typename A>
struct State {
    A v;
    int64_t i;  // argument index (ARG kinds), -1 = empty
};

template <int K, typename A>
__device__ __forceinline__ State<A> init_state() {
    State<A> s;
    s.i = -1;
    s.v = A(0);
    if constexpr (std::is_floating_point<A>::value) {
        if (K == K_MAX) s.v = -INFINITY;
        if (K == K_MIN) s.v = INFINITY;
    } else {
        if (K == K_MAX) s.v = INT64_MIN;
        if (K == K_MIN) s.v = INT64_MAX;
    }
    return s;
}

// Fold element v (index idx, visited in increasing order within a lane).
template <int K, typename A>
__device__ __forceinline__ void update(State<A>& s, A v, int64_t idx) {
    if (K == K_SUM) {
        s.v = s.v + v;
    } else if (K == K_MAX) {
        if constexpr (std::is_same<A, float>::value) s.v = fmax_nan(s.v, v);  // NaN sticks once seen
        else s.v = (v > s.v || v != v) ? v : s.v;
    } else if (K == K_MIN) {
        if constexpr (std::is_same<A, float>::value) s.v = fmin_nan(s.v, v);
        else s.v = (v < s.v || v != v) ? v : s.v;
    } else {
        const bool better = (K == K_ARGMAX) ? (v > s.v) : (v < s.v);
        const bool take = s.i < 0 || (s.v == s.v && (better || v != v));
        if (take) {
            s.v = v;
            s.i = idx;
        }
    }
}

// Fold N consecutive elements f[0..N) with indices base..base+N-1 (sum,
// max, min; arg kinds use ArgVec below).
template <int K, int N>
__device__ __forceinline__ void update_vec(State<float>& s, const float* f, int64_t base) {
#pragma unroll
    for (int j = 0; j < N; j++) update<K, float>(s, f[j], base + j);
}

// Combine two partial states; ties and NaN resolve to the lower index.
template <int K, typename A>
__device__ __forceinline__ State<A> combine(State<A> a, State<A> b) {
    if (K == K_SUM) {
        a.v = a.v + b.v;
        return a;
    } else if (K == K_MAX) {
        a.v = (b.v > a.v || b.v != b.v) ? b.v : a.v;
        return a;
    } else if (K == K_MIN) {
        a.v = (b.v < a.v || b.v != b.v) ? b.v : a.v;
        return a;
    } else {
        if (b.i < 0) return a;
        if (a.i < 0) return b;
        const bool an = a.v != a.v, bn = b.v != b.v;
        if (an || bn) {
            if (an && bn) return a.i < b.i ? a : b;
            return an ? a : b;
        }
        const bool b_better = (K == K_ARGMAX) ? (b.v > a.v) : (b.v < a.v);
        if (b_better || (b.v == a.v && b.i < a.i)) return b;
        return a;
    }
}

template <int K, typename A>
__device__ __forceinline__ State<A> warp_combine(State<A> s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        State<A> t;
        t.v = __shfl_xor_sync(0xffffffffu, s.v, o);
        t.i = __shfl_xor_sync(0xffffffffu, s.i, o);
        // Keep the combine order fixed: lower lane is the left operand.
        s = ((threadIdx.x & 31) & o) ? combine<K, A>(t, s) : combine<K, A>(s, t);
    }
    return s;
}

}  // namespace
}  // namespace tadma_b200
