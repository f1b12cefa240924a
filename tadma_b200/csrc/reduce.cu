// reduce.cu - reduction engine (sm_100a): sum / mean / max / min / argmax /
// argmin / sum-of-squares / rms along one axis.
//
// Replaces ReduceNode + ReduceKernel (kernels/Reduce.hpp:10-71), which moves
// the reduced axis to dim 0 with transpose<D,0> and runs one block per output
// element: a strided per-thread fold, then a shared-memory tree with a
// __syncthreads per level.  For a middle axis the lanes of a warp read
// addresses one row-stride apart (uncoalesced), and fp16 accumulates in fp16.
//
// Here the input is folded to [outer, R, inner] (layout.hpp) and:
// * ROW path (reduced axis contiguous, e.g. sum<-1>): one warp per output
//   row, 16-byte loads (4 x fp32 / 8 x 16-bit) with 4 loads in flight per
//   lane, fp32 accumulation, a 5-step shuffle butterfly;
// * COL path (reduced axis strided, inner contiguous, e.g. mean<1> of
//   [32,4096,4096]): a CTA owns 32 x VEC adjacent output columns; its 8 warps
//   split R (rows w, w+8, ...), each lane reading 16 contiguous bytes per row
//   so every warp load is a fully used 512-byte run; partials combine through
//   shared memory in warp order;
// * SPLIT (ROW or COL) when few outputs share a long reduced axis: several
//   CTAs per output reduce fixed chunks into a workspace, a second pass
//   combines the chunk partials in order; the COL split hands every CTA of
//   one resident wave the same number of rows (a CTA's share may end in one
//   column tile and go on in the next), so no SM waits on a second wave or
//   on a neighbour with one CTA more;
// * GENERIC path: any other layout / dtype, one warp per output element.
// Every path assigns elements to lanes and combines partials in a fixed
// order, so results are deterministic run to run.
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "layout.hpp"
#include "ops.cuh"
#include "reduce_state.cuh"

namespace tadma_b200 {
namespace {

enum Post { P_NONE = 0, P_MEAN = 1, P_RMS = 2 };

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

struct RedParams {
    const char* in;
    char* out;
    int32_t in_dtype, out_dtype;
    int32_t pre_op, square, post, kind;
    int64_t R;               // reduced extent
    int64_t r_stride;        // input stride along the reduced axis
    int64_t nrows;           // ROW: output count; COL: outer extent
    int64_t inner;           // COL: inner extent
    int64_t in_row_stride;   // ROW: input stride between outputs; COL: outer stride
    int64_t out_row_stride;  // ROW: output stride; COL: outer stride
    // GENERIC: folded kept dims
    int32_t krank, pad;
    int64_t kdims[TADMA_MAX_RANK];
    DivMod kdm[TADMA_MAX_RANK];
    int64_t kin[TADMA_MAX_RANK];
    int64_t kout[TADMA_MAX_RANK];
    // split-R (two-pass) reductions
    int64_t splits;  // CTAs per row (ROW) / partial slots per column tile (COL)
    int64_t chunk;   // ROW: reduced-axis elements per split
    // COL split: `ctas` CTAs share the `units` = tiles x nrows x R
    // (tile, row) pairs evenly, in tile-major order
    int64_t units, tiles, ctas, tile_cols;
    void* partials;  // State<float> workspace
    // row operand (reduce_rowop_kernel): element x of row r becomes
    // op1(x, m_r) before the pre-op, m_r = rop[r * rop_row_stride], or imm1
    // when rop is null
    const char* rop;
    int32_t rop_dtype, op1;
    int64_t rop_row_stride;
    double imm1;
    PostChain pc;  // applied to each reduced value before its store (n = 0: none)
};

// Element pre-op (fused unary and/or square).  PRE = false: the call has
// neither, and the fast kernels are instantiated without the per-element test.
template <bool PRE = true, typename A>
__device__ __forceinline__ A prep(const RedParams& p, A v) {
    if constexpr (PRE) {
        if (p.pre_op != TADMA_OP_COPY) v = unary(p.pre_op, v);
        if (p.square) v = sq(v);
    }
    return v;
}

template <int K, typename A>
__device__ __forceinline__ void finish(const RedParams& p, const State<A>& s, int64_t off) {
    if (K == K_ARGMAX || K == K_ARGMIN) {
        store_from(p.out, p.out_dtype, off, (int64_t)(s.i < 0 ? 0 : s.i));
        return;
    }
    A v = s.v;
    if constexpr (std::is_floating_point<A>::value) {
        if (p.post == P_MEAN) v = v / (A)p.R;
        else if (p.post == P_RMS) v = sqrt(v / (A)p.R);
    } else {
        if (p.post == P_MEAN) v = p.R ? v / p.R : 0;  // integer mean (x / Dim(D), Tensor.hpp:448)
    }
    if (p.pc.n) v = apply_post<A>(p.pc, v);
    store_from(p.out, p.out_dtype, off, v);
}

// 16-byte vector of T -> VEC floats
template <typename T>
struct Vec;
template <>
struct Vec<float> {
    static constexpr int N = 4;
    static __device__ __forceinline__ void cvt(uint4 r, float* f) {
        f[0] = __uint_as_float(r.x);
        f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z);
        f[3] = __uint_as_float(r.w);
    }
};
template <>
struct Vec<__half> {
    static constexpr int N = 8;
    static __device__ __forceinline__ void cvt(uint4 r, float* f) { unpack8(r, TADMA_F16, f); }
};
template <>
struct Vec<__nv_bfloat16> {
    static constexpr int N = 8;
    static __device__ __forceinline__ void cvt(uint4 r, float* f) { unpack8(r, TADMA_BF16, f); }
};

template <typename T>
__device__ __forceinline__ float ld1(const T* p) {
    if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float*>(p);
    else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
    else return __bfloat162float(*p);
}

// Per-lane arg-reduction over 16-byte vectors.  Each vector costs its N - 1
// NaN-propagating max/min ops, one "beats the best" test and the selects
// that keep the best vector's value, vector index and raw bits; the element
// index inside the winning vector is found once, in resolve().  A vector
// beats the best when its extreme is strictly better, or when it holds the
// first NaN (NaN counts as the extreme and sticks), so ties keep the
// earlier vector and, within it, the first matching element.
template <int K, typename T, int N>
struct ArgVec {
    float v;
    int64_t vi;  // vector index of the best, -1 = none yet
    uint4 raw;

    __device__ __forceinline__ void init() {
        v = (K == K_ARGMAX) ? -INFINITY : INFINITY;
        vi = -1;
        raw = make_uint4(0, 0, 0, 0);
    }
    __device__ __forceinline__ void add(const uint4& r, const float* f, int64_t vidx) {
        float m = f[0];
#pragma unroll
        for (int j = 1; j < N; j++) m = (K == K_ARGMAX) ? fmax_nan(m, f[j]) : fmin_nan(m, f[j]);
        const bool take = ((K == K_ARGMAX) ? (m > v) : (m < v)) || (m != m && v == v);
        v = take ? m : v;
        vi = take ? vidx : vi;
        raw.x = take ? r.x : raw.x;
        raw.y = take ? r.y : raw.y;
        raw.z = take ? r.z : raw.z;
        raw.w = take ? r.w : raw.w;
    }
    // tf: the element transform the reduction applied (its pre-op).
    template <typename TF>
    __device__ __forceinline__ State<float> resolve(const TF& tf) const {
        State<float> s;
        s.v = v;
        s.i = -1;
        if (vi < 0) return s;
        float f[N];
        Vec<T>::cvt(raw, f);
        int jj = 0;
#pragma unroll
        for (int j = N - 1; j >= 0; j--) {
            const float x = tf(f[j]);
            if (v != v ? x != x : x == v) jj = j;
        }
        s.i = vi * N + jj;
        return s;
    }
};

// -------------------------------------------------------------- ROW path --

template <typename T, int K, bool PRE>
__global__ void __launch_bounds__(THREADS) reduce_row_kernel(const __grid_constant__ RedParams p, int vec) {
    pdl_begin();
    constexpr int N = Vec<T>::N;
    constexpr int UNR = 4;
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    for (int64_t row = gw; row < p.nrows; row += nw) {
        const T* x = reinterpret_cast<const T*>(p.in) + row * p.in_row_stride;
        State<float> s = init_state<K, float>();
        int64_t done = 0;
        if (vec) {
            constexpr bool ARG = K == K_ARGMAX || K == K_ARGMIN;
            ArgVec<K, T, N> av;
            if constexpr (ARG) av.init();
            const int64_t nv = p.R / N;
            for (int64_t i0 = lane; i0 < nv; i0 += 32 * UNR) {
                uint4 r[UNR];
#pragma unroll
                for (int u = 0; u < UNR; u++)
                    if (i0 + 32 * u < nv) r[u] = ld_stream_v4(x + (i0 + 32 * u) * N);
#pragma unroll
                for (int u = 0; u < UNR; u++) {
                    if (i0 + 32 * u < nv) {
                        float f[N];
                        Vec<T>::cvt(r[u], f);
#pragma unroll
                        for (int j = 0; j < N; j++) f[j] = prep<PRE>(p, f[j]);
                        if constexpr (ARG) av.add(r[u], f, i0 + 32 * u);
                        else update_vec<K, N>(s, f, (i0 + 32 * u) * N);
                    }
                }
            }
            if constexpr (ARG) s = av.resolve([&](float x) { return prep<PRE>(p, x); });
            done = nv * N;
        }
        for (int64_t i = done + lane; i < p.R; i += 32) update<K, float>(s, prep<PRE>(p, ld1(x + i * p.r_stride)), i);
        s = warp_combine<K, float>(s);
        if (lane == 0) finish<K, float>(p, s, row * p.out_row_stride);
    }
}

// ------------------------------------------------- ROW path, row operand --
//
// A chain reduction whose chain is op1(x, m) [then a unary op] [then a
// square], with m one value per output row (a per-row tensor or an
// immediate): the row variance sum((x - mean)^2), the softmax denominator
// sum(exp(x - max)), scaled sums.  tadma_b200_reduce_chain sends those here
// instead of its interpreter: the same warp-per-row loop as
// reduce_row_kernel, with each op dispatched once per 16-byte vector (the op
// bodies of the element-wise engine, so the chain's values are bit-identical).

template <int N>
__device__ __forceinline__ void rowop_vec(const RedParams& p, float m, float (&f)[N]) {
#define TADMA_ROWOP_B(OPC)                                                         \
    case OPC:                                                                      \
        _Pragma("unroll") for (int j = 0; j < N; j++) f[j] = binary(OPC, f[j], m, 0.0f); \
        break;
    switch (p.op1) {
        TADMA_ROWOP_B(TADMA_OP_ADD)
        TADMA_ROWOP_B(TADMA_OP_SUB)
        TADMA_ROWOP_B(TADMA_OP_MUL)
        TADMA_ROWOP_B(TADMA_OP_DIV)
        TADMA_ROWOP_B(TADMA_OP_RSUB)
        TADMA_ROWOP_B(TADMA_OP_RDIV)
        TADMA_ROWOP_B(TADMA_OP_MAX)
        TADMA_ROWOP_B(TADMA_OP_MIN)
    default:
        break;
    }
#undef TADMA_ROWOP_B
#define TADMA_ROWOP_U(OPC)                                                         \
    case OPC:                                                                      \
        _Pragma("unroll") for (int j = 0; j < N; j++) f[j] = unary(OPC, f[j]);    \
        break;
    switch (p.pre_op) {
    case TADMA_OP_COPY:
        break;
        TADMA_ROWOP_U(TADMA_OP_EXP)
        TADMA_ROWOP_U(TADMA_OP_ABS)
        TADMA_ROWOP_U(TADMA_OP_NEG)
        TADMA_ROWOP_U(TADMA_OP_SQRT)
    default:
#pragma unroll
        for (int j = 0; j < N; j++) f[j] = unary(p.pre_op, f[j]);
        break;
    }
#undef TADMA_ROWOP_U
    if (p.square) {
#pragma unroll
        for (int j = 0; j < N; j++) f[j] = sq(f[j]);
    }
}

__device__ __forceinline__ float rowop_one(const RedParams& p, float m, float x) {
    float f[1] = {x};
    rowop_vec<1>(p, m, f);
    return f[0];
}

template <typename T, int K>
__global__ void __launch_bounds__(THREADS) reduce_rowop_kernel(const __grid_constant__ RedParams p, int vec) {
    pdl_begin();
    constexpr int N = Vec<T>::N;
    constexpr int UNR = 4;
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    __shared__ uint4 ring_s[THREADS / 32][2][UNR][32];  // 32 KB: 2 stages x UNR vectors x 32 lanes per warp
    uint4 (*ring)[UNR][32] = ring_s[threadIdx.x >> 5];
    for (int64_t row = gw; row < p.nrows; row += nw) {
        const T* x = reinterpret_cast<const T*>(p.in) + row * p.in_row_stride;
        const float m = p.rop ? load_as<float>(p.rop, p.rop_dtype, row * p.rop_row_stride) : __double2float_rn(p.imm1);
        State<float> s = init_state<K, float>();
        int64_t done = 0;
        if (vec) {
            constexpr bool ARG = K == K_ARGMAX || K == K_ARGMIN;
            ArgVec<K, T, N> av;
            if constexpr (ARG) av.init();
            const int64_t nv = p.R / N;
            // The lane's vectors i0, i0 + 32, ... go through its slots of the
            // warp's two-stage ring with cp.async, the next group's copies in
            // flight while this group runs its chain (exp, division) and
            // folds; the lane reads back only what it copied.
            auto issue = [&](int64_t g0, int st) {
#pragma unroll
                for (int u = 0; u < UNR; u++)
                    if (g0 + 32 * u < nv) cp_async16(&ring[st][u][lane], x + (g0 + 32 * u) * N);
                cp_async_commit();
            };
            int st = 0;
            issue(lane, 0);
            for (int64_t i0 = lane; i0 < nv; i0 += 32 * UNR, st ^= 1) {
                issue(i0 + 32 * UNR, st ^ 1);
                cp_async_wait<1>();
#pragma unroll
                for (int u = 0; u < UNR; u++) {
                    if (i0 + 32 * u < nv) {
                        const uint4 r = ring[st][u][lane];
                        float f[N];
                        Vec<T>::cvt(r, f);
                        rowop_vec<N>(p, m, f);
                        if constexpr (ARG) av.add(r, f, i0 + 32 * u);
                        else update_vec<K, N>(s, f, (i0 + 32 * u) * N);
                    }
                }
            }
            cp_async_wait<0>();  // the last (empty) group, before the ring's reuse
            if constexpr (ARG) s = av.resolve([&](float v) { return rowop_one(p, m, v); });
            done = nv * N;
        }
        for (int64_t i = done + lane; i < p.R; i += 32) update<K, float>(s, rowop_one(p, m, ld1(x + i)), i);
        s = warp_combine<K, float>(s);
        if (lane == 0) finish<K, float>(p, s, row * p.out_row_stride);
    }
}

// -------------------------------------------------------------- COL path --

// The CTA of a COL split whose share holds (tile, row) pair x: CTA c starts
// at pair c * units / ctas.
__host__ __device__ __forceinline__ int64_t col_cta_of(int64_t x, int64_t units, int64_t ctas) {
    return ((x + 1) * ctas + units - 1) / units - 1;
}

// Rows [rbeg, rend) of column tile `tile` of outer index o: warps take rows
// rbeg + w, rbeg + w + 8, ..., lanes 32 x VEC adjacent columns; the warp
// partials combine in warp order, then go to the output or (SPLIT) to
// partial slot k of the tile.
template <typename T, int K, int VEC, bool SPLIT, bool PRE>
__device__ __forceinline__ void col_segment(const RedParams& p, int64_t o, int64_t tile, int64_t rbeg, int64_t rend, int64_t k,
                                            State<float> (&part)[WARPS][32 * VEC]) {
    constexpr int COLS = 32 * VEC;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t col0 = tile * COLS + lane * VEC;
    const T* base = reinterpret_cast<const T*>(p.in) + o * p.in_row_stride;
    State<float> s[VEC];
#pragma unroll
    for (int j = 0; j < VEC; j++) s[j] = init_state<K, float>();
    if (col0 < p.inner) {
        constexpr int UNR = 4;
        for (int64_t r0 = rbeg + w; r0 < rend; r0 += WARPS * UNR) {
            if constexpr (VEC > 1) {
                uint4 v[UNR];
#pragma unroll
                for (int u = 0; u < UNR; u++)
                    if (r0 + WARPS * u < rend) v[u] = ld_stream_v4(base + (r0 + WARPS * u) * p.r_stride + col0);
#pragma unroll
                for (int u = 0; u < UNR; u++) {
                    if (r0 + WARPS * u < rend) {
                        float f[Vec<T>::N];
                        Vec<T>::cvt(v[u], f);
#pragma unroll
                        for (int j = 0; j < VEC; j++) update<K, float>(s[j], prep<PRE>(p, f[j]), r0 + WARPS * u);
                    }
                }
            } else {
                float v[UNR];
#pragma unroll
                for (int u = 0; u < UNR; u++)
                    if (r0 + WARPS * u < rend) v[u] = ld1(base + (r0 + WARPS * u) * p.r_stride + col0);
#pragma unroll
                for (int u = 0; u < UNR; u++)
                    if (r0 + WARPS * u < rend) update<K, float>(s[0], prep<PRE>(p, v[u]), r0 + WARPS * u);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < VEC; j++) part[w][lane * VEC + j] = s[j];
    __syncthreads();
    for (int c = threadIdx.x; c < COLS; c += THREADS) {
        const int64_t col = tile * COLS + c;
        if (col < p.inner) {
            State<float> t = part[0][c];
#pragma unroll
            for (int ww = 1; ww < WARPS; ww++) t = combine<K, float>(t, part[ww][c]);
            if constexpr (SPLIT) {
                reinterpret_cast<State<float>*>(p.partials)[(o * p.splits + k) * p.inner + col] = t;
            } else {
                finish<K, float>(p, t, o * p.out_row_stride + col);
            }
        }
    }
    __syncthreads();
}

// SPLIT: a 1-D grid of p.ctas CTAs; CTA c reduces (tile, row) pairs
// [c U / P, (c + 1) U / P) of the tile-major sequence (U = p.units, P =
// p.ctas), one segment per tile its share touches, each into the slot given
// by its rank among the tile's CTAs.  Otherwise blockIdx.x is the tile and
// blockIdx.y walks the outer index.
template <typename T, int K, int VEC, bool SPLIT, bool PRE>
__global__ void __launch_bounds__(THREADS) reduce_col_kernel(const __grid_constant__ RedParams p) {
    pdl_begin();
    __shared__ State<float> part[WARPS][32 * VEC];
    if constexpr (SPLIT) {
        const int64_t U = p.units, P = p.ctas, c = blockIdx.x;
        const int64_t ue = (c + 1) * U / P;
        for (int64_t u = c * U / P; u < ue;) {
            const int64_t tb = u / p.R, rbeg = u - tb * p.R;
            const int64_t rend = rbeg + (ue - u) < p.R ? rbeg + (ue - u) : p.R;
            const int64_t o = tb / p.tiles;
            col_segment<T, K, VEC, true, PRE>(p, o, tb - o * p.tiles, rbeg, rend, c - col_cta_of(tb * p.R, U, P), part);
            u += rend - rbeg;
        }
    } else {
        for (int64_t o = blockIdx.y; o < p.nrows; o += gridDim.y)
            col_segment<T, K, VEC, false, PRE>(p, o, blockIdx.x, 0, p.R, 0, part);
    }
}

// ----------------------------------------------------- split-R (two-pass) --
//
// Few output rows with a long reduced axis leave most SMs idle on the one-warp-
// (or one-CTA-) per-output paths.  Pass 1 gives each output `splits` CTAs, each
// reducing one fixed chunk of R into a State in a workspace; pass 2 combines
// the partials of an output in chunk order.  Chunks and combine order depend
// only on (R, splits), so results are deterministic.

template <typename T, int K, bool PRE>
__global__ void __launch_bounds__(THREADS) reduce_row_split_kernel(const __grid_constant__ RedParams p, int vec) {
    pdl_begin();
    constexpr int N = Vec<T>::N;
    constexpr int UNR = 4;
    __shared__ State<float> sh[WARPS];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int64_t row = blockIdx.y, g = blockIdx.x;
    const int64_t r0 = g * p.chunk;
    const int64_t r1 = r0 + p.chunk < p.R ? r0 + p.chunk : p.R;
    const T* x = reinterpret_cast<const T*>(p.in) + row * p.in_row_stride;
    State<float> s = init_state<K, float>();
    int64_t done = r0;
    if (vec) {  // chunk % N == 0, so every chunk starts 16-byte aligned
        constexpr bool ARG = K == K_ARGMAX || K == K_ARGMIN;
        ArgVec<K, T, N> av;
        if constexpr (ARG) av.init();
        const int64_t v0 = r0 / N, v1 = r1 / N;
        for (int64_t i0 = v0 + threadIdx.x; i0 < v1; i0 += THREADS * UNR) {
            uint4 r[UNR];
#pragma unroll
            for (int u = 0; u < UNR; u++)
                if (i0 + THREADS * u < v1) r[u] = ld_stream_v4(x + (i0 + THREADS * u) * N);
#pragma unroll
            for (int u = 0; u < UNR; u++) {
                if (i0 + THREADS * u < v1) {
                    float f[N];
                    Vec<T>::cvt(r[u], f);
#pragma unroll
                    for (int j = 0; j < N; j++) f[j] = prep<PRE>(p, f[j]);
                    if constexpr (ARG) av.add(r[u], f, i0 + THREADS * u);
                    else update_vec<K, N>(s, f, (i0 + THREADS * u) * N);
                }
            }
        }
        if constexpr (ARG) s = av.resolve([&](float x) { return prep<PRE>(p, x); });
        done = v1 * N;
    }
    for (int64_t i = done + threadIdx.x; i < r1; i += THREADS) update<K, float>(s, prep<PRE>(p, ld1(x + i * p.r_stride)), i);
    s = warp_combine<K, float>(s);
    if (lane == 0) sh[w] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        State<float> t = sh[0];
#pragma unroll
        for (int ww = 1; ww < WARPS; ww++) t = combine<K, float>(t, sh[ww]);
        reinterpret_cast<State<float>*>(p.partials)[row * p.splits + g] = t;
    }
}

// Pass 2 of the ROW split: one warp per output row.
template <int K>
__global__ void __launch_bounds__(THREADS) reduce_row_finish_kernel(const __grid_constant__ RedParams p) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    const State<float>* part = reinterpret_cast<const State<float>*>(p.partials);
    for (int64_t row = gw; row < p.nrows; row += nw) {
        State<float> s = init_state<K, float>();
        for (int64_t g = lane; g < p.splits; g += 32) s = combine<K, float>(s, part[row * p.splits + g]);
        s = warp_combine<K, float>(s);
        if (lane == 0) finish<K, float>(p, s, row * p.out_row_stride);
    }
}

// Pass 2 of the COL split: one thread per output column of an outer index.
template <int K>
__global__ void __launch_bounds__(THREADS) reduce_col_finish_kernel(const __grid_constant__ RedParams p) {
    pdl_begin();
    const State<float>* part = reinterpret_cast<const State<float>*>(p.partials);
    const int64_t total = p.nrows * p.inner;
    for (int64_t idx = (int64_t)blockIdx.x * THREADS + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * THREADS) {
        const int64_t o = idx / p.inner, col = idx - o * p.inner;
        // the CTAs whose shares cover this column's tile, in row order
        const int64_t x = (o * p.tiles + col / p.tile_cols) * p.R;
        const int64_t n = col_cta_of(x + p.R - 1, p.units, p.ctas) - col_cta_of(x, p.units, p.ctas) + 1;
        State<float> t = init_state<K, float>();
        for (int64_t g = 0; g < n; g++) t = combine<K, float>(t, part[(o * p.splits + g) * p.inner + col]);
        finish<K, float>(p, t, o * p.out_row_stride + col);
    }
}

// ---------------------------------------------------------- GENERIC path --

template <typename A, int K>
__global__ void __launch_bounds__(THREADS) reduce_generic_kernel(const __grid_constant__ RedParams p) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    for (int64_t o = gw; o < p.nrows; o += nw) {
        uint64_t e = (uint64_t)o;
        int64_t ioff = 0, ooff = 0;
        for (int d = p.krank - 1; d >= 1; d--) {
            uint64_t q, r;
            p.kdm[d].divmod(e, q, r);
            ioff += (int64_t)r * p.kin[d];
            ooff += (int64_t)r * p.kout[d];
            e = q;
        }
        ioff += (int64_t)e * p.kin[0];
        ooff += (int64_t)e * p.kout[0];
        State<A> s = init_state<K, A>();
        for (int64_t r = lane; r < p.R; r += 32) {
            A v = load_as<A>(p.in, p.in_dtype, ioff + r * p.r_stride);
            update<K, A>(s, prep(p, v), r);
        }
        s = warp_combine<K, A>(s);
        if (lane == 0) {
            finish<K, A>(p, s, ooff);
        }
    }
}

// ------------------------------------------------------------- host side --

int blocks_per_sm(const void* fn) {
    static std::mutex mu;
    static std::unordered_map<const void*, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(fn);
    if (it != cache.end()) return it->second;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, THREADS, 0) != cudaSuccess || nb <= 0) nb = 1;
    cache[fn] = nb;
    return nb;
}

int grid_for(const void* fn, int64_t want) {
    int64_t cap = (int64_t)sm_count() * blocks_per_sm(fn);
    if (want < 1) want = 1;
    return (int)(want < cap ? want : cap);
}

template <typename T, int K, bool PRE>
int launch_fast(int path, const RedParams& p, bool vec, cudaStream_t s) {
    if (path == 0) {
        if (p.splits > 1) {
            (void)launch_pdl(reduce_row_split_kernel<T, K, PRE>, dim3(dim3((unsigned)p.splits, (unsigned)p.nrows)), dim3(THREADS), 0, s, p, vec ? 1 : 0);
            const void* fn = (const void*)reduce_row_finish_kernel<K>;
            (void)launch_pdl(reduce_row_finish_kernel<K>, dim3(grid_for(fn, (p.nrows + WARPS - 1) / WARPS)), dim3(THREADS), 0, s, p);
        } else {
            const void* fn = (const void*)reduce_row_kernel<T, K, PRE>;
            int grid = grid_for(fn, (p.nrows + WARPS - 1) / WARPS);
            (void)launch_pdl(reduce_row_kernel<T, K, PRE>, dim3(grid), dim3(THREADS), 0, s, p, vec ? 1 : 0);
        }
    } else {
        constexpr int VEC = Vec<T>::N;
        int64_t tiles = vec ? (p.inner + 32 * VEC - 1) / (32 * VEC) : (p.inner + 31) / 32;
        if (tiles > 0x7fffffff) return fail(TADMA_ERR_UNSUPPORTED, "reduce: too many column tiles");
        dim3 grid((unsigned)tiles, (unsigned)(p.nrows < 65535 ? p.nrows : 65535), 1);
        if (p.splits > 1) {
            const dim3 g1((unsigned)p.ctas);
            if (vec) (void)launch_pdl(reduce_col_kernel<T, K, VEC, true, PRE>, g1, dim3(THREADS), 0, s, p);
            else (void)launch_pdl(reduce_col_kernel<T, K, 1, true, PRE>, g1, dim3(THREADS), 0, s, p);
            const void* fn = (const void*)reduce_col_finish_kernel<K>;
            (void)launch_pdl(reduce_col_finish_kernel<K>, dim3(grid_for(fn, (p.nrows * p.inner + THREADS - 1) / THREADS)), dim3(THREADS), 0, s, p);
        } else {
            if (vec) (void)launch_pdl(reduce_col_kernel<T, K, VEC, false, PRE>, dim3(grid), dim3(THREADS), 0, s, p);
            else (void)launch_pdl(reduce_col_kernel<T, K, 1, false, PRE>, dim3(grid), dim3(THREADS), 0, s, p);
        }
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_reduce launch");
}

template <typename T, bool PRE>
int launch_fast_kind_pre(int kind, int path, const RedParams& p, bool vec, cudaStream_t s) {
    switch (kind) {
    case K_SUM: return launch_fast<T, K_SUM, PRE>(path, p, vec, s);
    case K_MAX: return launch_fast<T, K_MAX, PRE>(path, p, vec, s);
    case K_MIN: return launch_fast<T, K_MIN, PRE>(path, p, vec, s);
    case K_ARGMAX: return launch_fast<T, K_ARGMAX, PRE>(path, p, vec, s);
    default: return launch_fast<T, K_ARGMIN, PRE>(path, p, vec, s);
    }
}

template <typename T>
int launch_fast_kind(int kind, int path, const RedParams& p, bool vec, cudaStream_t s) {
    if (p.pre_op != TADMA_OP_COPY || p.square) return launch_fast_kind_pre<T, true>(kind, path, p, vec, s);
    return launch_fast_kind_pre<T, false>(kind, path, p, vec, s);
}

// The COL split kernel of (T, kind, vector path, pre-op) and the number of
// its CTAs resident at once on the device.
template <typename T, bool PRE>
const void* col_split_fn(int kind, bool vec) {
    constexpr int V = Vec<T>::N;
    switch (kind) {
    case K_SUM: return vec ? (const void*)reduce_col_kernel<T, K_SUM, V, true, PRE> : (const void*)reduce_col_kernel<T, K_SUM, 1, true, PRE>;
    case K_MAX: return vec ? (const void*)reduce_col_kernel<T, K_MAX, V, true, PRE> : (const void*)reduce_col_kernel<T, K_MAX, 1, true, PRE>;
    case K_MIN: return vec ? (const void*)reduce_col_kernel<T, K_MIN, V, true, PRE> : (const void*)reduce_col_kernel<T, K_MIN, 1, true, PRE>;
    case K_ARGMAX:
        return vec ? (const void*)reduce_col_kernel<T, K_ARGMAX, V, true, PRE> : (const void*)reduce_col_kernel<T, K_ARGMAX, 1, true, PRE>;
    default:
        return vec ? (const void*)reduce_col_kernel<T, K_ARGMIN, V, true, PRE> : (const void*)reduce_col_kernel<T, K_ARGMIN, 1, true, PRE>;
    }
}

int64_t col_split_capacity(int dt, int kind, bool vec, bool pre) {
    const void* fn;
    switch (dt) {
    case TADMA_F32: fn = pre ? col_split_fn<float, true>(kind, vec) : col_split_fn<float, false>(kind, vec); break;
    case TADMA_F16: fn = pre ? col_split_fn<__half, true>(kind, vec) : col_split_fn<__half, false>(kind, vec); break;
    default: fn = pre ? col_split_fn<__nv_bfloat16, true>(kind, vec) : col_split_fn<__nv_bfloat16, false>(kind, vec); break;
    }
    return (int64_t)sm_count() * blocks_per_sm(fn);
}

template <typename A>
int launch_generic(int kind, const RedParams& p, cudaStream_t s) {
    const void* fn;
    switch (kind) {
    case K_SUM: fn = (const void*)reduce_generic_kernel<A, K_SUM>; break;
    case K_MAX: fn = (const void*)reduce_generic_kernel<A, K_MAX>; break;
    case K_MIN: fn = (const void*)reduce_generic_kernel<A, K_MIN>; break;
    case K_ARGMAX: fn = (const void*)reduce_generic_kernel<A, K_ARGMAX>; break;
    default: fn = (const void*)reduce_generic_kernel<A, K_ARGMIN>; break;
    }
    int grid = grid_for(fn, (p.nrows + WARPS - 1) / WARPS);
    switch (kind) {
    case K_SUM: (void)launch_pdl(reduce_generic_kernel<A, K_SUM>, dim3(grid), dim3(THREADS), 0, s, p); break;
    case K_MAX: (void)launch_pdl(reduce_generic_kernel<A, K_MAX>, dim3(grid), dim3(THREADS), 0, s, p); break;
    case K_MIN: (void)launch_pdl(reduce_generic_kernel<A, K_MIN>, dim3(grid), dim3(THREADS), 0, s, p); break;
    case K_ARGMAX: (void)launch_pdl(reduce_generic_kernel<A, K_ARGMAX>, dim3(grid), dim3(THREADS), 0, s, p); break;
    default: (void)launch_pdl(reduce_generic_kernel<A, K_ARGMIN>, dim3(grid), dim3(THREADS), 0, s, p); break;
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_reduce launch");
}

// Split plans: how many CTAs share one output's reduced axis (1 = no split).
// ROW: split when fewer than 16 warps per SM would be busy and R is long.
void plan_row_split(RedParams& p, int64_t R, int64_t sm) {
    p.splits = 1;
    if (p.nrows >= 16 * sm || R < 16384 || p.nrows > 65535) return;
    int64_t g = (4 * sm + p.nrows - 1) / p.nrows;
    if (g > R / 4096) g = R / 4096;
    if (g > 65535) g = 65535;
    if (g < 2) return;
    int64_t chunk = ((R + g - 1) / g + 7) / 8 * 8;  // multiple of every vector width
    p.chunk = chunk;
    p.splits = (R + chunk - 1) / chunk;
}

// COL: split when fewer than 2 CTAs per SM would be busy and R is long:
// one resident wave of the split kernel (`capacity` CTAs, at least 256 rows
// each) shares the tiles' rows evenly.  splits: the partial slots per tile,
// the most CTAs one tile's R rows can span.
void plan_col_split(RedParams& p, int64_t R, int64_t cols_per_cta, int64_t sm, int64_t capacity) {
    p.splits = 1;
    const int64_t tiles = (p.inner + cols_per_cta - 1) / cols_per_cta;
    const int64_t ctas = tiles * p.nrows;
    if (ctas >= 2 * sm || R < 2048 || p.nrows > 65535) return;
    const int64_t U = ctas * R;
    int64_t P = capacity;
    if (P > U / 256) P = U / 256;
    if (P <= ctas) return;
    p.units = U;
    p.tiles = tiles;
    p.tile_cols = cols_per_cta;
    p.ctas = P;
    p.splits = (P + ctas - 1) / ctas + 1;
}

int64_t split_workspace_bytes(const RedParams& p, int path) {
    if (p.splits <= 1) return 0;
    const int64_t states = path == 0 ? p.nrows * p.splits : p.nrows * p.splits * p.inner;
    return states * (int64_t)sizeof(State<float>);
}

int dispatch_fast(int dt, int kind, int path, const RedParams& p, bool vec, cudaStream_t s) {
    switch (dt) {
    case TADMA_F32: return launch_fast_kind<float>(kind, path, p, vec, s);
    case TADMA_F16: return launch_fast_kind<__half>(kind, path, p, vec, s);
    default: return launch_fast_kind<__nv_bfloat16>(kind, path, p, vec, s);
    }
}

// Runs a fast path; a split plan gets a stream-ordered workspace for its
// partials (cudaMallocAsync / cudaFreeAsync on the call's stream, so calls on
// different streams never share it).
// A fixed scratch buffer given by the no-allocation entry point (null for
// tadma_b200_reduce, which allocates its workspace per call).
struct FixedScratch {
    void* ptr = nullptr;
    int64_t bytes = 0;
};

int run_fast(int dt, int kind, int path, RedParams& p, bool vec, cudaStream_t s, const FixedScratch& fixed) {
    const int64_t ws = split_workspace_bytes(p, path);
    if (ws == 0) return dispatch_fast(dt, kind, path, p, vec, s);
    if (fixed.ptr) {
        if (ws > fixed.bytes) {
            // Fewer splits, so the partials fit the static scratch; with room
            // for fewer than two, the reduction runs in one pass (no scratch).
            const int64_t per_split = ws / p.splits;
            const int64_t g = fixed.bytes / per_split;
            if (path == 1) {
                // COL: fewer CTAs, so that a tile's rows span at most g of them
                const int64_t ctas = p.tiles * p.nrows;
                if (g < 3) {
                    p.splits = 1;
                    return dispatch_fast(dt, kind, path, p, vec, s);
                }
                if (p.ctas > (g - 1) * ctas) p.ctas = (g - 1) * ctas;
                p.splits = (p.ctas + ctas - 1) / ctas + 1;
            } else {
                if (g < 2) {
                    p.splits = 1;
                    return dispatch_fast(dt, kind, path, p, vec, s);
                }
                p.chunk = ((p.R + g - 1) / g + 7) / 8 * 8;  // a multiple of every vector width
                p.splits = (p.R + p.chunk - 1) / p.chunk;
            }
        }
        p.partials = fixed.ptr;
        return dispatch_fast(dt, kind, path, p, vec, s);
    }
    void* buf = nullptr;
    cudaError_t e = workspace_alloc(&buf, (size_t)ws, s);
    if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_reduce workspace");
    p.partials = buf;
    int rc = dispatch_fast(dt, kind, path, p, vec, s);
    e = cudaFreeAsync(buf, s);
    if (rc == TADMA_OK && e != cudaSuccess) return cuda_fail(e, "tadma_b200_reduce workspace free");
    return rc;
}

int reduce_impl(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op, const tadma_tensor* out,
                void* stream, const FixedScratch& fixed);

int reduce_impl(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op, const tadma_tensor* out,
                void* stream, const FixedScratch& fixed) {
    std::string err = check_tensor(in, "in");
    if (err.empty()) err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (op < TADMA_REDUCE_SUM || op > TADMA_REDUCE_RMS) return fail(TADMA_ERR_INVALID, "unknown reduce op");
    if (in->rank < 1) return fail(TADMA_ERR_INVALID, "reduce needs rank >= 1");
    const int ax = axis < 0 ? axis + in->rank : axis;
    if (ax < 0 || ax >= in->rank) return fail(TADMA_ERR_INVALID, "axis out of range");
    const bool keep = out->rank == in->rank;
    if (!keep && out->rank != in->rank - 1) return fail(TADMA_ERR_INVALID, "out rank must be in rank or in rank - 1");
    for (int d = 0, k = 0; d < in->rank; d++) {
        if (d == ax) {
            if (keep && out->dims[d] != 1) return fail(TADMA_ERR_INVALID, "out dims[axis] must be 1");
            if (keep) k++;
            continue;
        }
        if (out->dims[k] != in->dims[d]) return fail(TADMA_ERR_INVALID, "out dims do not match in dims");
        k++;
    }
    const bool arg = op == TADMA_REDUCE_ARGMAX || op == TADMA_REDUCE_ARGMIN;
    if (arg && out->dtype != TADMA_I64 && out->dtype != TADMA_I32)
        return fail(TADMA_ERR_INVALID, "argmax/argmin output must be int64 or int32");
    if (pre_op != TADMA_OP_COPY && !(pre_op > 0 && pre_op <= TADMA_OP_NOT))
        return fail(TADMA_ERR_INVALID, "pre_op must be a unary op code");
    const int64_t R = in->dims[ax];
    if (R == 0 && op != TADMA_REDUCE_SUM && op != TADMA_REDUCE_SUMSQ)
        return fail(TADMA_ERR_INVALID, "empty reduction has no identity for this op");
    if (numel(out) == 0) return TADMA_OK;

    // Kept dims, folded jointly for in and out.
    int64_t kd[TADMA_MAX_RANK], ks[2][TADMA_MAX_RANK];
    int kr = 0;
    for (int d = 0; d < in->rank; d++) {
        if (d == ax) continue;
        kd[kr] = in->dims[d];
        ks[0][kr] = in->strides[d];
        ks[1][kr] = out->strides[keep ? d : (d < ax ? d : d - 1)];
        kr++;
    }
    Folded f = fold(kr, kd, ks, 2);

    RedParams p{};
    p.in = (const char*)in->data;
    p.out = (char*)out->data;
    p.in_dtype = in->dtype;
    p.out_dtype = out->dtype;
    p.pre_op = pre_op;
    p.square = (op == TADMA_REDUCE_SUMSQ || op == TADMA_REDUCE_RMS);
    p.post = op == TADMA_REDUCE_MEAN ? P_MEAN : (op == TADMA_REDUCE_RMS ? P_RMS : P_NONE);
    int kind;
    switch (op) {
    case TADMA_REDUCE_MAX: kind = K_MAX; break;
    case TADMA_REDUCE_MIN: kind = K_MIN; break;
    case TADMA_REDUCE_ARGMAX: kind = K_ARGMAX; break;
    case TADMA_REDUCE_ARGMIN: kind = K_ARGMIN; break;
    default: kind = K_SUM; break;
    }
    p.kind = kind;
    p.R = R;
    p.r_stride = in->strides[ax];
    cudaStream_t s = (cudaStream_t)stream;

    const int dt = in->dtype;
    const bool fast_dt = dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16;
    const int es = dtype_size(dt);
    const int last = f.rank - 1;
    const bool in_aligned = ((uintptr_t)in->data % 16) == 0;
    if (fast_dt && R > 1 && p.r_stride == 1 && f.rank == 1) {
        // ROW
        p.nrows = f.dims[0];
        p.in_row_stride = f.strides[0][0];
        p.out_row_stride = f.strides[1][0];
        const int N = 16 / es;
        bool vec = in_aligned && R >= N && (p.nrows == 1 || (p.in_row_stride * es) % 16 == 0);
        plan_row_split(p, R, sm_count());
        return run_fast(dt, kind, 0, p, vec, s, fixed);
    }
    if (fast_dt && R > 1 && p.r_stride != 1 && f.rank <= 2 && f.strides[0][last] == 1 && f.strides[1][last] == 1 &&
        f.dims[last] > 1) {
        // COL
        p.inner = f.dims[last];
        p.nrows = f.rank == 2 ? f.dims[0] : 1;
        p.in_row_stride = f.rank == 2 ? f.strides[0][0] : 0;
        p.out_row_stride = f.rank == 2 ? f.strides[1][0] : 0;
        const int N = 16 / es;
        bool vec = in_aligned && p.inner % N == 0 && (p.r_stride * es) % 16 == 0 && (p.in_row_stride * es) % 16 == 0;
        plan_col_split(p, R, vec ? 32 * N : 32, sm_count(),
                       col_split_capacity(dt, kind, vec, p.pre_op != TADMA_OP_COPY || p.square));
        return run_fast(dt, kind, 1, p, vec, s, fixed);
    }
    // GENERIC
    p.krank = f.rank;
    p.nrows = 1;
    for (int d = 0; d < f.rank; d++) {
        p.kdims[d] = f.dims[d];
        p.kdm[d] = DivMod((uint64_t)f.dims[d]);
        p.kin[d] = f.strides[0][d];
        p.kout[d] = f.strides[1][d];
        p.nrows *= f.dims[d];
    }
    const bool int_acc = !dtype_is_float(dt) && pre_op == TADMA_OP_COPY && op != TADMA_REDUCE_RMS;
    if (int_acc) return launch_generic<int64_t>(kind, p, s);
    return launch_generic<double>(kind, p, s);
}

}  // namespace
}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_reduce(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op,
                                 const tadma_tensor* out, void* stream) {
    return reduce_impl(op, in, axis, pre_op, out, stream, FixedScratch{});
}

// ------------------------------------------------- no-allocation variant --
//
// Some callers cannot call cudaMalloc: a serving process whose memory pool
// has claimed the device's HBM up front (any further allocation fails), a
// real-time path that forbids the latency of an allocator call, or a host
// that only lends this library the buffers it passes in.
// tadma_b200_reduce_noalloc serves them: the partials of split reductions
// live in this file-scope device array (every GPU that loads the library
// holds it until the process exits) instead of a per-call workspace.

constexpr int64_t NOALLOC_SCRATCH_BYTES = 2 << 20;  // 2 MiB
static __device__ __align__(256) unsigned char g_reduce_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_reduce_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
static int noalloc_scratch(void** ptr) {
    static std::mutex mu;
    static std::vector<void*> cache;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_reduce_noalloc: cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if ((int)cache.size() <= dev) cache.resize(dev + 1, nullptr);
    if (!cache[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_reduce_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_reduce_noalloc: cudaGetSymbolAddress");
        if (!p) return fail(TADMA_ERR_CUDA, "tadma_b200_reduce_noalloc: cudaGetSymbolAddress returned a null address");
        cache[dev] = p;
    }
    *ptr = cache[dev];
    return TADMA_OK;
}

extern "C" int tadma_b200_reduce_noalloc(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op,
                                         const tadma_tensor* out, void* stream) {
    FixedScratch fixed;
    int rc = noalloc_scratch(&fixed.ptr);
    if (rc != TADMA_OK) return rc;
    fixed.bytes = NOALLOC_SCRATCH_BYTES;
    return reduce_impl(op, in, axis, pre_op, out, stream, fixed);
}

namespace tadma_b200 {

// The row-operand reduction (reduce_rowop_kernel) for tadma_b200_reduce_chain:
// out = reduce over `axis` of sq(pre(op1(in, m))), m = rop broadcast along
// the axis (or imm1 when rop is null), `shape` the broadcast execution shape
// of in and rop.  Only the unsplit ROW layout is taken: the reduced axis
// contiguous in `in`, the kept dims of in, rop and out folding to one.  Any
// other layout returns TADMA_ERR_UNSUPPORTED without recording an error, and
// the caller runs its general kernel instead.
int reduce_rowop(int32_t op, const int64_t* shape, int32_t rank, int32_t ax, const tadma_tensor* in, int32_t op1,
                 const tadma_tensor* rop, double imm1, int32_t pre_op, int32_t square, const tadma_instr* post,
                 int32_t n_post, const tadma_tensor* out, cudaStream_t s) {
    const int dt = in->dtype;
    if (!(dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16)) return TADMA_ERR_UNSUPPORTED;
    const int64_t R = shape[ax];
    if (R < 2 || in->dims[ax] != R || in->strides[ax] != 1) return TADMA_ERR_UNSUPPORTED;
    if (rop && rop->dims[ax] != 1 && rop->strides[ax] != 0) return TADMA_ERR_UNSUPPORTED;
    const bool keep = out->rank == rank;
    int64_t kd[TADMA_MAX_RANK], ks[3][TADMA_MAX_RANK];
    int kr = 0;
    for (int d = 0; d < rank; d++) {
        if (d == ax) continue;
        kd[kr] = shape[d];
        ks[0][kr] = in->dims[d] == 1 ? 0 : in->strides[d];
        ks[1][kr] = out->strides[keep ? d : (d < ax ? d : d - 1)];
        ks[2][kr] = !rop || rop->dims[d] == 1 ? 0 : rop->strides[d];
        kr++;
    }
    int64_t nrows = 1, in_rs = 0, out_rs = 0, rop_rs = 0;
    if (kr > 0) {
        Folded f = fold(kr, kd, ks, 3);
        if (f.rank != 1) return TADMA_ERR_UNSUPPORTED;
        nrows = f.dims[0];
        in_rs = f.strides[0][0];
        out_rs = f.strides[1][0];
        rop_rs = f.strides[2][0];
    }
    RedParams p{};
    p.in = (const char*)in->data;
    p.out = (char*)out->data;
    p.in_dtype = dt;
    p.out_dtype = out->dtype;
    p.pre_op = pre_op;
    p.square = square;
    p.post = op == TADMA_REDUCE_MEAN ? P_MEAN : (op == TADMA_REDUCE_RMS ? P_RMS : P_NONE);
    int kind;
    switch (op) {
    case TADMA_REDUCE_MAX: kind = K_MAX; break;
    case TADMA_REDUCE_MIN: kind = K_MIN; break;
    case TADMA_REDUCE_ARGMAX: kind = K_ARGMAX; break;
    case TADMA_REDUCE_ARGMIN: kind = K_ARGMIN; break;
    default: kind = K_SUM; break;
    }
    p.kind = kind;
    p.R = R;
    p.r_stride = 1;
    p.nrows = nrows;
    p.in_row_stride = in_rs;
    p.out_row_stride = out_rs;
    p.rop = rop ? (const char*)rop->data : nullptr;
    p.rop_dtype = rop ? rop->dtype : TADMA_F32;
    p.rop_row_stride = rop_rs;
    p.op1 = op1;
    p.imm1 = imm1;
    p.pc.n = n_post;
    for (int i = 0; i < n_post; i++) p.pc.prog[i] = post[i];
    plan_row_split(p, R, sm_count());
    if (p.splits > 1) return TADMA_ERR_UNSUPPORTED;  // few long rows: the general kernel's split-free path
    const int es = dtype_size(dt);
    const bool vec = ((uintptr_t)in->data % 16) == 0 && R >= 16 / es && (nrows == 1 || (in_rs * es) % 16 == 0);
    auto go = [&](auto kern) {
        const int grid = grid_for((const void*)kern, (p.nrows + WARPS - 1) / WARPS);
        (void)launch_pdl(kern, dim3(grid), dim3(THREADS), 0, s, p, vec ? 1 : 0);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_reduce_chain launch");
    };
    auto by_kind = [&](auto tag) {
        using T = decltype(tag);
        switch (kind) {
        case K_SUM: return go(reduce_rowop_kernel<T, K_SUM>);
        case K_MAX: return go(reduce_rowop_kernel<T, K_MAX>);
        case K_MIN: return go(reduce_rowop_kernel<T, K_MIN>);
        case K_ARGMAX: return go(reduce_rowop_kernel<T, K_ARGMAX>);
        default: return go(reduce_rowop_kernel<T, K_ARGMIN>);
        }
    };
    if (dt == TADMA_F32) return by_kind(float{});
    if (dt == TADMA_F16) return by_kind(__half{});
    return by_kind(__nv_bfloat16{});
}

}  // namespace tadma_b200
