// eltwise.cu - fused element-wise / broadcast engine (sm_100a).
//
// Replaces the reference's lazy-node executor: EltwiseNode / CombineToNode /
// CombineNode / InplaceNode (Kernels.hpp:16-53) run through CUDAHIPExecutor
// (Node.hpp:25-48): one scalar element per thread, 512-thread blocks, a 32-bit
// index and an int64 div/mod per dimension per element.  MergeNodes
// (Node.hpp:189-224) composes node lambdas into one kernel; here a fused
// chain is a short instruction list (tadma_instr) evaluated in registers.
//
// Design:
// * the joint layout of out and inputs is folded (layout.hpp); typical
//   launches become rank 1 (streaming) or rank 2 (row broadcast);
// * vector path: each thread step handles V = 8 consecutive elements with
//   16-byte loads/stores (2 x 16 B for fp32, 1 x 16 B for 16-bit types); an
//   operand whose innermost stride is 0 is loaded once and splatted;
//   operands with no broadcast stream through with evict-first hints;
// * one contiguous chunk per CTA (U = 2 vector steps per thread, 1 with 3-4
//   operands, loaded before any compute) and as many CTAs as chunks, so the
//   block scheduler balances the SMs;
// * any other layout takes the scalar path (SU elements per thread, DivMod
//   index decomposition, still 64-bit safe);
// * the chain is uniform across the grid (kernel parameters), so the
//   per-instruction switch is a uniform branch amortised over 8 elements.
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"
#include "layout.hpp"
#include "ops.cuh"
#include "reduce_state.cuh"

namespace tadma_b200 {
namespace {

constexpr int V = 8;        // elements per vector step
// Vector steps in flight per thread: 2, or 1 with 3-4 operands (their
// registers would otherwise halve the resident warps).
template <int NIN>
constexpr int vec_steps() { return NIN >= 3 ? 1 : 2; }
constexpr int THREADS = 256;

struct Operand {
    const char* base;
    int32_t dtype;
    int32_t inner_bcast;  // innermost folded stride is 0
    int32_t streaming;    // no stride-0 dim: evict-first loads
    int32_t pad;
    int64_t stride[TADMA_MAX_RANK];
};

struct ChainParams {
    int32_t rank;
    int32_t n_instr;
    int32_t out_dtype;
    int32_t idx32;  // 1: every element index is below 2^32 (32-bit quotients);
                    // 2: also every operand offset below 2^31 (32-bit offset sums)
    int64_t start;  // first element (scalar tail launch)
    int64_t n;      // element count (scalar path) / vector count (vector path)
    int64_t dims[TADMA_MAX_RANK];
    DivMod dm[TADMA_MAX_RANK];
    char* out;
    int64_t out_stride[TADMA_MAX_RANK];
    Operand in[TADMA_MAX_INPUTS];
    tadma_instr prog[TADMA_MAX_INSTR];
    float scale;  // affine program: the MUL immediate, rounded to fp32
};

// Program selector of a kernel instance: the run-time interpreter (precise or
// fast math) or a compile-time affine + activation chain act(x * s + b).
constexpr int PROG_INTERP = 0;
constexpr int PROG_INTERP_FAST = 1;
constexpr int ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2, ACT_SIGMOID = 3, ACT_TANH = 4;
constexpr int affine_prog(int act, bool fast, bool mul, bool add) {
    return 0x100 | (act << 4) | (fast ? 4 : 0) | (mul ? 2 : 0) | (add ? 1 : 0);
}

template <typename C>
__device__ __forceinline__ C imm_as(double v);
template <>
__device__ __forceinline__ float imm_as<float>(double v) { return __double2float_rn(v); }
template <>
__device__ __forceinline__ double imm_as<double>(double v) { return v; }
template <>
__device__ __forceinline__ int64_t imm_as<int64_t>(double v) { return f2i(v); }

// Operand selection: static indices only, so `val` stays in registers.
template <typename C, int NIN, int W>
__device__ __forceinline__ void select(int sel, double imm, const C (&val)[NIN > 0 ? NIN : 1][W], C (&dst)[W]) {
    if (sel < 0 || sel >= NIN) {
        C s = imm_as<C>(imm);
#pragma unroll
        for (int j = 0; j < W; j++) dst[j] = s;
        return;
    }
#pragma unroll
    for (int k = 0; k < NIN; k++) {
        if (sel == k) {
#pragma unroll
            for (int j = 0; j < W; j++) dst[j] = val[k][j];
        }
    }
}

// One dispatch per instruction per vector: every case carries its own
// unrolled W-element loop with the op code as a compile-time constant, so the
// scalar op bodies (ops.cuh) constant-fold their switch.
#define TADMA_UCASE(OPC)                                        \
    case OPC: {                                                 \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = unary<FAST>(OPC, acc[j]); \
    } break;
#define TADMA_BCASE(OPC)                                        \
    case OPC: {                                                 \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = binary(OPC, acc[j], b[j], c[j]); \
    } break;
#define TADMA_RCASE(DT)                                         \
    case DT: {                                                  \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = round_to(acc[j], DT); \
    } break;

template <typename C, int W, bool FAST>
__device__ __forceinline__ void unary_vec(int op, C (&acc)[W]) {
    switch (op) {
        TADMA_UCASE(TADMA_OP_NEG)
        TADMA_UCASE(TADMA_OP_ABS)
        TADMA_UCASE(TADMA_OP_EXP)
        TADMA_UCASE(TADMA_OP_SQRT)
        TADMA_UCASE(TADMA_OP_RELU)
        TADMA_UCASE(TADMA_OP_SIGMOID)
        TADMA_UCASE(TADMA_OP_TANH)
        TADMA_UCASE(TADMA_OP_GELU)
        TADMA_UCASE(TADMA_OP_NOT)
    default: {
#pragma unroll
        for (int j = 0; j < W; j++) acc[j] = unary<FAST>(op, acc[j]);
    } break;
    }
}

template <typename C, int W>
__device__ __forceinline__ void binary_vec(int op, C (&acc)[W], const C (&b)[W], const C (&c)[W]) {
    switch (op) {
        TADMA_BCASE(TADMA_OP_ADD)
        TADMA_BCASE(TADMA_OP_SUB)
        TADMA_BCASE(TADMA_OP_MUL)
        TADMA_BCASE(TADMA_OP_DIV)
        TADMA_BCASE(TADMA_OP_POW)
        TADMA_BCASE(TADMA_OP_RSUB)
        TADMA_BCASE(TADMA_OP_RDIV)
        TADMA_BCASE(TADMA_OP_MAX)
        TADMA_BCASE(TADMA_OP_MIN)
        TADMA_BCASE(TADMA_OP_EQ)
        TADMA_BCASE(TADMA_OP_NE)
        TADMA_BCASE(TADMA_OP_LT)
        TADMA_BCASE(TADMA_OP_GT)
        TADMA_BCASE(TADMA_OP_LE)
        TADMA_BCASE(TADMA_OP_GE)
        TADMA_BCASE(TADMA_OP_AND)
        TADMA_BCASE(TADMA_OP_OR)
        TADMA_BCASE(TADMA_OP_XOR)
        TADMA_BCASE(TADMA_OP_LAND)
        TADMA_BCASE(TADMA_OP_LOR)
        TADMA_BCASE(TADMA_OP_WHERE)
    default:
        break;
    }
}

template <typename C, int W>
__device__ __forceinline__ void round_vec(int dt, C (&acc)[W]) {
    switch (dt) {
        TADMA_RCASE(TADMA_F16)
        TADMA_RCASE(TADMA_BF16)
        TADMA_RCASE(TADMA_I64)
        TADMA_RCASE(TADMA_I32)
        TADMA_RCASE(TADMA_U8)
        TADMA_RCASE(TADMA_BOOL)
        TADMA_RCASE(TADMA_I8)
        TADMA_RCASE(TADMA_F32)
    default:
        break;  // F64: nothing to round
    }
}

template <typename C, int NIN, int W, bool FAST>
__device__ __forceinline__ void run_chain(const ChainParams& p, C (&acc)[W], const C (&val)[NIN > 0 ? NIN : 1][W]) {
    for (int i = 0; i < p.n_instr; i++) {
        const tadma_instr& I = p.prog[i];
        const int op = I.op;
        if (op < 32) {
            if (op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM) {
                C s = imm_as<C>(I.imm);
#pragma unroll
                for (int j = 0; j < W; j++) acc[j] = s;
            } else if (op != TADMA_OP_COPY) {
                unary_vec<C, W, FAST>(op, acc);
            }
        } else {
            C b[W], c[W];
            select<C, NIN, W>(I.b, I.imm, val, b);
            if (op == TADMA_OP_WHERE) {
                select<C, NIN, W>(I.c, I.imm, val, c);
            } else {
#pragma unroll
                for (int j = 0; j < W; j++) c[j] = b[j];
            }
            binary_vec<C, W>(op, acc, b, c);
        }
        if (I.round_dtype >= 0) {
            if constexpr (sizeof(C) == 4) {
                if (I.round_dtype != TADMA_F32 && I.round_dtype != TADMA_F64) round_vec<C, W>(I.round_dtype, acc);
            } else {
                round_vec<C, W>(I.round_dtype, acc);
            }
        }
    }
}

template <int ACT, bool FAST>
__device__ __forceinline__ float activation(float v) {
    if constexpr (ACT == ACT_GELU) return unary<FAST>(TADMA_OP_GELU, v);
    else if constexpr (ACT == ACT_RELU) return unary<FAST>(TADMA_OP_RELU, v);
    else if constexpr (ACT == ACT_SIGMOID) return unary<FAST>(TADMA_OP_SIGMOID, v);
    else if constexpr (ACT == ACT_TANH) return unary<FAST>(TADMA_OP_TANH, v);
    else return v;
}

// Runs the kernel's program on W elements.  The affine program uses the very
// op bodies the interpreter uses (__fmul_rn, __fadd_rn, unary<FAST>), so both
// paths give identical bits for the same chain.
template <typename C, int NIN, int W, int PROG>
__device__ __forceinline__ void program(const ChainParams& p, C (&acc)[W], const C (&val)[NIN > 0 ? NIN : 1][W]) {
    if constexpr (PROG == PROG_INTERP || PROG == PROG_INTERP_FAST) {
        run_chain<C, NIN, W, PROG == PROG_INTERP_FAST>(p, acc, val);
    } else {
        constexpr int ACT = (PROG >> 4) & 0xf;
        constexpr bool FAST = (PROG & 4) != 0, MUL = (PROG & 2) != 0, ADD = (PROG & 1) != 0;
        static_assert(std::is_same<C, float>::value && (!ADD || NIN == 2));
#pragma unroll
        for (int j = 0; j < W; j++) {
            float v = acc[j];
            if constexpr (MUL) v = __fmul_rn(v, p.scale);
            if constexpr (ADD) v = __fadd_rn(v, val[NIN > 1 ? 1 : 0][j]);
            acc[j] = activation<ACT, FAST>(v);
        }
    }
}

// ------------------------------------------------------- vector load/store --

template <typename C>
__device__ __forceinline__ C from_f(float f);
template <>
__device__ __forceinline__ float from_f<float>(float f) { return f; }
template <>
__device__ __forceinline__ double from_f<double>(float f) { return (double)f; }
template <>
__device__ __forceinline__ int64_t from_f<int64_t>(float f) { return f2i(f); }

template <typename C>
__device__ __forceinline__ void load_vec(const Operand& o, int64_t off, C (&v)[V]) {
    if (o.inner_bcast) {
        C s = load_as<C>(o.base, o.dtype, off);
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = s;
        return;
    }
    const char* p = o.base + off * dtype_size(o.dtype);
    switch (o.dtype) {
    case TADMA_F32: {
        uint4 a = o.streaming ? ld_stream_v4(p) : ld_v4(p);
        uint4 b = o.streaming ? ld_stream_v4(p + 16) : ld_v4(p + 16);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = from_f<C>(__uint_as_float(w[j]));
        break;
    }
    case TADMA_F16:
    case TADMA_BF16: {
        uint4 a = o.streaming ? ld_stream_v4(p) : ld_v4(p);
        float f[8];
        unpack8(a, o.dtype, f);
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = from_f<C>(f[j]);
        break;
    }
    case TADMA_U8:
    case TADMA_BOOL:
    case TADMA_I8: {
        // 8 one-byte elements in one 8-byte load; values as load_as gives them
        const uint2 a = o.streaming ? __ldcs(reinterpret_cast<const uint2*>(p)) : *reinterpret_cast<const uint2*>(p);
#pragma unroll
        for (int j = 0; j < V; j++) {
            const uint32_t byte = ((j < 4 ? a.x : a.y) >> (8 * (j & 3))) & 0xffu;
            const int32_t iv = o.dtype == TADMA_I8 ? (int32_t)(int8_t)byte : o.dtype == TADMA_BOOL ? (byte != 0u) : (int32_t)byte;
            v[j] = (C)iv;
        }
        break;
    }
    default: {
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = load_as<C>(o.base, o.dtype, off + j);
        break;
    }
    }
}

// The byte store_from writes for a one-byte dtype.
template <typename C>
__device__ __forceinline__ uint32_t to_byte(C v, int dt) {
    if (dt == TADMA_BOOL) return v != C(0) ? 1u : 0u;
    int64_t i;
    if constexpr (std::is_integral<C>::value) i = v;
    else i = f2i(v);
    return (uint32_t)(uint8_t)i;
}

template <typename C>
__device__ __forceinline__ float to_f(C v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<double>(double v) { return __double2float_rn(v); }
template <>
__device__ __forceinline__ float to_f<int64_t>(int64_t v) { return __ll2float_rn(v); }

template <typename C>
__device__ __forceinline__ void store_vec(char* base, int dt, int64_t off, const C (&v)[V]) {
    char* p = base + off * dtype_size(dt);
    switch (dt) {
    case TADMA_F32: {
        if constexpr (sizeof(C) == 4) {
            uint4 a = make_uint4(__float_as_uint(to_f(v[0])), __float_as_uint(to_f(v[1])), __float_as_uint(to_f(v[2])), __float_as_uint(to_f(v[3])));
            uint4 b = make_uint4(__float_as_uint(to_f(v[4])), __float_as_uint(to_f(v[5])), __float_as_uint(to_f(v[6])), __float_as_uint(to_f(v[7])));
            st_stream_v4(p, a);
            st_stream_v4(p + 16, b);
            break;
        }
    }
        [[fallthrough]];
    default:
        if (dt == TADMA_F16 || dt == TADMA_BF16) {
            float f[8];
#pragma unroll
            for (int j = 0; j < V; j++) f[j] = to_f(v[j]);
            st_stream_v4(p, pack8(f, dt));
        } else if (dt == TADMA_U8 || dt == TADMA_BOOL || dt == TADMA_I8) {
            uint2 w = make_uint2(0u, 0u);
#pragma unroll
            for (int j = 0; j < V; j++) {
                const uint32_t b = to_byte<C>(v[j], dt) << (8 * (j & 3));
                if (j < 4) w.x |= b;
                else w.y |= b;
            }
            __stcs(reinterpret_cast<uint2*>(p), w);
        } else {
#pragma unroll
            for (int j = 0; j < V; j++) store_from(base, dt, off + j, v[j]);
        }
        break;
    }
}

// Narrow operands (every input 1 or 2 bytes wide, or an innermost broadcast
// of at most 4 bytes): one vector is kept as its raw 16-byte word and
// converted to fp32 only when it is computed, so a thread can hold 4 vectors
// of 2 operands in flight in 32 registers.
__device__ __forceinline__ uint4 load_raw_narrow(const Operand& o, int64_t off) {
    if (o.inner_bcast) {
        // the element's raw bits (<= 4 bytes) in .x
        const char* q = o.base + off * dtype_size(o.dtype);
        const int es = dtype_size(o.dtype);
        const uint32_t bits = es == 4 ? *reinterpret_cast<const uint32_t*>(q)
                            : es == 2 ? (uint32_t)*reinterpret_cast<const uint16_t*>(q)
                                      : (uint32_t)*reinterpret_cast<const uint8_t*>(q);
        return make_uint4(bits, 0u, 0u, 0u);
    }
    const char* q = o.base + off * dtype_size(o.dtype);
    if (dtype_size(o.dtype) == 2) return o.streaming ? ld_stream_v4(q) : ld_v4(q);
    const uint2 a = o.streaming ? __ldcs(reinterpret_cast<const uint2*>(q)) : *reinterpret_cast<const uint2*>(q);
    return make_uint4(a.x, a.y, 0u, 0u);
}

// fp32 value of one narrow element given its raw bits (as load_as<float>).
__device__ __forceinline__ float narrow_value(uint32_t bits, int dt) {
    switch (dt) {
    case TADMA_F32: return __uint_as_float(bits);
    case TADMA_F16: return __half2float(__ushort_as_half((unsigned short)bits));
    case TADMA_BF16: return __uint_as_float(bits << 16);
    case TADMA_I32: return __int2float_rn((int32_t)bits);
    case TADMA_U8: return (float)(bits & 0xffu);
    case TADMA_BOOL: return (bits & 0xffu) != 0u ? 1.0f : 0.0f;
    case TADMA_I8: return (float)(int8_t)(bits & 0xffu);
    }
    return 0.0f;
}

__device__ __forceinline__ void cvt_raw_narrow(const Operand& o, uint4 r, float (&v)[V]) {
    if (o.inner_bcast) {
        const float x = narrow_value(r.x, o.dtype);
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = x;
    } else if (o.dtype == TADMA_F16 || o.dtype == TADMA_BF16) {
        unpack8(r, o.dtype, v);
    } else {
#pragma unroll
        for (int j = 0; j < V; j++) {
            const uint32_t byte = ((j < 4 ? r.x : r.y) >> (8 * (j & 3))) & 0xffu;
            v[j] = o.dtype == TADMA_I8 ? (float)(int8_t)byte : o.dtype == TADMA_BOOL ? (byte != 0u ? 1.0f : 0.0f) : (float)byte;
        }
    }
}

// ----------------------------------------------------------------- kernels --

template <int NIN>
__device__ __forceinline__ void offsets(const ChainParams& p, uint64_t e, int64_t& oo, int64_t (&io)[NIN > 0 ? NIN : 1]) {
    oo = 0;
#pragma unroll
    for (int k = 0; k < NIN; k++) io[k] = 0;
    if (p.idx32 == 2) {
        // 32-bit quotients and offset sums: the host checked that every
        // operand's largest offset (all strides >= 0) is below 2^31.
        uint32_t e32 = (uint32_t)e, o32 = 0, i32[NIN > 0 ? NIN : 1];
#pragma unroll
        for (int k = 0; k < NIN; k++) i32[k] = 0;
        for (int d = p.rank - 1; d >= 1; d--) {
            const uint32_t q = p.dm[d].div32(e32), r = e32 - q * (uint32_t)p.dm[d].d;
            o32 += r * (uint32_t)p.out_stride[d];
#pragma unroll
            for (int k = 0; k < NIN; k++) i32[k] += r * (uint32_t)p.in[k].stride[d];
            e32 = q;
        }
        oo = (int64_t)(o32 + e32 * (uint32_t)p.out_stride[0]);
#pragma unroll
        for (int k = 0; k < NIN; k++) io[k] = (int64_t)(i32[k] + e32 * (uint32_t)p.in[k].stride[0]);
        return;
    }
    if (p.idx32) {
        // Same walk with 32-bit quotients (the host sets idx32 only when the
        // element count is below 2^32); offsets stay 64-bit.
        uint32_t e32 = (uint32_t)e;
        for (int d = p.rank - 1; d >= 1; d--) {
            const uint32_t q = p.dm[d].div32(e32), r = e32 - q * (uint32_t)p.dm[d].d;
            oo += (int64_t)r * p.out_stride[d];
#pragma unroll
            for (int k = 0; k < NIN; k++) io[k] += (int64_t)r * p.in[k].stride[d];
            e32 = q;
        }
        e = e32;
    } else {
        for (int d = p.rank - 1; d >= 1; d--) {
            uint64_t q, r;
            p.dm[d].divmod(e, q, r);
            oo += (int64_t)r * p.out_stride[d];
#pragma unroll
            for (int k = 0; k < NIN; k++) io[k] += (int64_t)r * p.in[k].stride[d];
            e = q;
        }
    }
    oo += (int64_t)e * p.out_stride[0];
#pragma unroll
    for (int k = 0; k < NIN; k++) io[k] += (int64_t)e * p.in[k].stride[0];
}

// Both kernels give each CTA one contiguous chunk of work and are launched
// with enough CTAs to cover the launch in one pass (the loop over chunks only
// runs past one iteration when the work needs more than 2^31 - 1 CTAs): the
// hardware block scheduler then balances SMs, where a persistent grid-stride
// loop measured 10-15 % slower on B200.
template <typename C, int NIN, int PROG>
__global__ void __launch_bounds__(THREADS) chain_vec_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int NI = NIN > 0 ? NIN : 1;
    constexpr int U = vec_steps<NIN>();
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        C val[U][NI][V];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NI];
                offsets<NIN>(p, (uint64_t)vi * V, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++) load_vec<C>(p.in[k], io[k], val[u][k]);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                C acc[V];
#pragma unroll
                for (int j = 0; j < V; j++) acc[j] = NIN > 0 ? val[u][0][j] : C(0);
                program<C, NIN, V, PROG>(p, acc, val[u]);
                store_vec<C>(p.out, p.out_dtype, oo[u], acc);
            }
        }
    }
}

// The narrow-operand variant of chain_vec_kernel (fp32 compute): raw words
// of U vectors per thread are loaded before any compute.
template <int NIN>
constexpr int narrow_steps() { return NIN >= 3 ? 2 : 4; }

template <int NIN, int PROG>
__global__ void __launch_bounds__(THREADS) chain_narrow_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int NI = NIN > 0 ? NIN : 1;
    constexpr int U = narrow_steps<NIN>();
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        uint4 raw[U][NI];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NI];
                offsets<NIN>(p, (uint64_t)vi * V, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++) raw[u][k] = load_raw_narrow(p.in[k], io[k]);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                float val[NI][V];
#pragma unroll
                for (int k = 0; k < NIN; k++) cvt_raw_narrow(p.in[k], raw[u][k], val[k]);
                float acc[V];
#pragma unroll
                for (int j = 0; j < V; j++) acc[j] = NIN > 0 ? val[0][j] : 0.0f;
                program<float, NIN, V, PROG>(p, acc, val);
                store_vec<float>(p.out, p.out_dtype, oo[u], acc);
            }
        }
    }
}

constexpr int SU = 4;  // elements per thread of the scalar kernel

template <typename C, int NIN, int PROG>
__global__ void __launch_bounds__(THREADS) chain_scalar_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int NI = NIN > 0 ? NIN : 1;
    for (int64_t chunk = blockIdx.x; p.start + chunk * (THREADS * SU) < p.n; chunk += gridDim.x) {
#pragma unroll
        for (int k = 0; k < SU; k++) {
            const int64_t e = p.start + chunk * (THREADS * SU) + k * THREADS + threadIdx.x;
            if (e >= p.n) break;
            int64_t oo, io[NI];
            offsets<NIN>(p, (uint64_t)e, oo, io);
            C val[NI][1];
#pragma unroll
            for (int q = 0; q < NIN; q++) val[q][0] = load_as<C>(p.in[q].base, p.in[q].dtype, io[q]);
            C acc[1] = {NIN > 0 ? val[0][0] : C(0)};
            program<C, NIN, 1, PROG>(p, acc, val);
            store_from(p.out, p.out_dtype, oo, acc[0]);
        }
    }
}

// ------------------------------------------------------ row-broadcast affine --
//
// y[r, c] = act(x[r, c] * s + b[c]) over a [rows, cols] layout (cols % 8 == 0)
// with a row-broadcast b: the bias-plus-activation pattern of config 2 and of
// every dense layer.  Each thread owns one 8-column vector of a tile of RB
// rows, so b is loaded and converted once per RB rows, no index division is
// needed, and all RB rows' loads are in flight before the first computes.
// x * s + b and the fast GELU polynomial run as packed fp32x2
// instructions (sm_100), every lane rounded as the scalar op would be, so the
// bits equal the generic path's (__fmul_rn, __fadd_rn, activation<ACT, FAST>).

struct AffineRowsParams {
    const char* x;
    const char* bias;
    char* out;
    int64_t rows, ncv;      // rows, 8-element column vectors
    int64_t x_rs, out_rs;   // row strides (elements)
    float scale;
};

template <typename T>
struct Raw8x {
    uint4 w[sizeof(T) == 4 ? 2 : 1];
};

template <typename T>
__device__ __forceinline__ void raw8_load(const T* p, Raw8x<T>& r, bool stream) {
    r.w[0] = stream ? ld_stream_v4(p) : ld_v4(p);
    if constexpr (sizeof(T) == 4) r.w[1] = stream ? ld_stream_v4(p + 4) : ld_v4(p + 4);
}

template <typename T>
__device__ __forceinline__ void raw8_cvt(const Raw8x<T>& r, float* f) {
    if constexpr (sizeof(T) == 4) {
        const uint32_t w[8] = {r.w[0].x, r.w[0].y, r.w[0].z, r.w[0].w, r.w[1].x, r.w[1].y, r.w[1].z, r.w[1].w};
#pragma unroll
        for (int j = 0; j < 8; j++) f[j] = __uint_as_float(w[j]);
    } else {
        unpack8(r.w[0], std::is_same<T, __half>::value ? TADMA_F16 : TADMA_BF16, f);
    }
}

template <typename T>
__device__ __forceinline__ void raw8_store(T* p, const float* f) {
    if constexpr (sizeof(T) == 4) {
        st_stream_v4(p, make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3])));
        st_stream_v4(p + 4, make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]), __float_as_uint(f[6]), __float_as_uint(f[7])));
    } else {
        st_stream_v4(p, pack8(f, std::is_same<T, __half>::value ? TADMA_F16 : TADMA_BF16));
    }
}

// gelu_fast on two lanes: the same operation sequence as gelu_fast (ops.cuh),
// gelu(x) = x / (1 + 2^(-w)), w = x (K1 + K3 x^2), with the polynomial, the
// sum and the final product packed (the sign of w folded into K1, K3).
__device__ __forceinline__ unsigned long long gelu_fast2(unsigned long long x) {
    constexpr float K1 = 2.0f * 0.7978845608f * 1.4426950408889634f;
    constexpr float K3 = K1 * 0.044715f;
    const unsigned long long nw = f2_mul(x, f2_fma(f2_pack(-K3, -K3), f2_mul(x, x), f2_pack(-K1, -K1)));
    float a, b;
    f2_unpack(nw, a, b);
    float d0, d1;
    f2_unpack(f2_add(f2_pack(ex2_approx(a), ex2_approx(b)), f2_pack(1.0f, 1.0f)), d0, d1);
    return f2_mul(x, f2_pack(rcp_approx(d0), rcp_approx(d1)));
}

template <typename XT, typename OT, int ACT>
__device__ __forceinline__ void affine_row_compute(const Raw8x<XT>& raw, const float (&b)[8],
                                                   const unsigned long long (&b2)[4], float scale, OT* dst) {
    constexpr bool FAST = sizeof(OT) == 2;  // same rule as the host: fp32 compute, 16-bit store
    float v[8];
    raw8_cvt<XT>(raw, v);
    if constexpr (ACT == ACT_NONE || (ACT == ACT_GELU && FAST)) {
        const unsigned long long s2 = f2_pack(scale, scale);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            unsigned long long x = f2_add(f2_mul(f2_pack(v[2 * j], v[2 * j + 1]), s2), b2[j]);
            if constexpr (ACT == ACT_GELU) x = gelu_fast2(x);
            f2_unpack(x, v[2 * j], v[2 * j + 1]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = activation<ACT, FAST>(__fadd_rn(__fmul_rn(v[j], scale), b[j]));
    }
    raw8_store<OT>(dst, v);
}

// One CTA per tile of RB consecutive rows x 256 column vectors, no loop: all
// RB rows' loads are issued before the first row computes, and the hardware
// block scheduler hands tiles to SMs as they free up (a persistent grid-stride
// loop measured 10-15 % slower on B200 for streaming copies: its fixed share of
// work per CTA leaves the slowest SMs finishing last).
template <typename XT>
constexpr int affine_rb() { return sizeof(XT) == 2 ? 8 : 4; }

template <typename XT, typename OT, int ACT>
__global__ void __launch_bounds__(THREADS) affine_rows_kernel(const __grid_constant__ AffineRowsParams p) {
    pdl_begin();
    constexpr int RB = affine_rb<XT>();
    // blockIdx.x = row tile * column blocks + column block: the column blocks
    // of one row tile are neighbours in launch order (one contiguous region).
    const int64_t ncb = (p.ncv + THREADS - 1) / THREADS;
    const int64_t tile = (int64_t)blockIdx.x / ncb;
    const int64_t cv = ((int64_t)blockIdx.x - tile * ncb) * THREADS + threadIdx.x;
    if (cv >= p.ncv) return;
    const int64_t r0 = tile * RB;
    const XT* xcol = reinterpret_cast<const XT*>(p.x) + cv * 8;
    OT* ocol = reinterpret_cast<OT*>(p.out) + cv * 8;
    Raw8x<XT> cur[RB];
#pragma unroll
    for (int u = 0; u < RB; u++)
        if (r0 + u < p.rows) raw8_load<XT>(xcol + (r0 + u) * p.x_rs, cur[u], true);
    float b[8];
    unsigned long long b2[4];
    {
        Raw8x<XT> rb;
        raw8_load<XT>(reinterpret_cast<const XT*>(p.bias) + cv * 8, rb, false);
        raw8_cvt<XT>(rb, b);
#pragma unroll
        for (int j = 0; j < 4; j++) b2[j] = f2_pack(b[2 * j], b[2 * j + 1]);
    }
#pragma unroll
    for (int u = 0; u < RB; u++)
        if (r0 + u < p.rows) affine_row_compute<XT, OT, ACT>(cur[u], b, b2, p.scale, ocol + (r0 + u) * p.out_rs);
}

// ------------------------------------------------------- contiguous typed --
//
// Every input of one float dtype TI with a contiguous innermost dim (no
// innermost broadcast), the output of float dtype TO, fp32 compute (residual
// adds, scalings, casts, copies into and out of strided views): loads,
// conversions and stores are compile-time and only the chain is interpreted.
// The generic kernels decode dtypes per vector, which cost ~170 instructions
// per 8 elements on a 16-bit add (ncu) and held it to 4.7 TB/s.

// Two vectors per thread: with the interpreter inlined once per vector, more
// would grow the kernel past what the instruction cache holds.
template <typename TI>
constexpr int typed_steps() { return 2; }

// Element offsets of vector vi: R1 (folded rank 1, every operand contiguous)
// needs no index decomposition; otherwise the folded dims are walked
// (outer-dim broadcasts and strided views; the innermost dim is contiguous).
template <int NIN, bool R1>
__device__ __forceinline__ void typed_offsets(const ChainParams& p, int64_t vi, int64_t& oo, int64_t (&io)[NIN]) {
    if constexpr (R1) {
        oo = vi * V;
#pragma unroll
        for (int k = 0; k < NIN; k++) io[k] = vi * V;
    } else {
        offsets<NIN>(p, (uint64_t)vi * V, oo, io);
    }
}

template <typename TI, typename TO, int NIN, bool FAST, bool R1>
__global__ void __launch_bounds__(THREADS) typed_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int U = typed_steps<TI>();
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        Raw8x<TI> raw[U][NIN];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NIN];
                typed_offsets<NIN, R1>(p, vi, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    raw8_load<TI>(reinterpret_cast<const TI*>(p.in[k].base) + io[k], raw[u][k], p.in[k].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                float val[NIN][V];
#pragma unroll
                for (int k = 0; k < NIN; k++) raw8_cvt<TI>(raw[u][k], val[k]);
                float acc[V];
#pragma unroll
                for (int j = 0; j < V; j++) acc[j] = val[0][j];
                run_chain<float, NIN, V, FAST>(p, acc, val);
                raw8_store<TO>(reinterpret_cast<TO*>(p.out) + oo[u], acc);
            }
        }
    }
}

// Single-instruction chains (every operator call of the eager API: a + b,
// x * s, a cast): the op is a compile-time constant as well, so no
// interpreter is inlined at all.  OP is ADD, SUB, MUL, DIV, RSUB, RDIV, MAX,
// MIN or COPY; IMM: the second operand is the immediate, else ins[1].
// Vectors per thread: 64 bytes of loads in flight for one 16-bit operand
// (4 x 16 B), as for an fp32 operand (2 x 32 B) or two 16-bit ones.
template <typename TI, int NIN>
constexpr int typed1_u() { return sizeof(TI) == 2 && NIN == 1 ? 4 : 2; }

template <typename TI, typename TO, int OP, bool IMM, bool R1>
__global__ void __launch_bounds__(THREADS) typed1_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int NIN = (OP == TADMA_OP_COPY || IMM) ? 1 : 2;
    constexpr int U = typed1_u<TI, NIN>();
    const float imm = __double2float_rn(p.prog[0].imm);
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        Raw8x<TI> raw[U][NIN];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NIN];
                typed_offsets<NIN, R1>(p, vi, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    raw8_load<TI>(reinterpret_cast<const TI*>(p.in[k].base) + io[k], raw[u][k], p.in[k].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if constexpr (OP == TADMA_OP_COPY && std::is_same<TI, TO>::value) {
                // A copy within one dtype moves the raw words (bit-exact).
                if (vi < p.n) {
                    TO* dst = reinterpret_cast<TO*>(p.out) + oo[u];
                    st_stream_v4(dst, raw[u][0].w[0]);
                    if constexpr (sizeof(TO) == 4) st_stream_v4(dst + 4, raw[u][0].w[1]);
                }
                continue;
            }
            if (vi < p.n) {
                float a[V], b[V];
                raw8_cvt<TI>(raw[u][0], a);
                if constexpr (NIN == 2) raw8_cvt<TI>(raw[u][NIN - 1], b);
#pragma unroll
                for (int j = 0; j < V; j++) {
                    if constexpr (OP != TADMA_OP_COPY) a[j] = binary(OP, a[j], IMM ? imm : b[j], 0.0f);
                }
                raw8_store<TO>(reinterpret_cast<TO*>(p.out) + oo[u], a);
            }
        }
    }
}

template <typename TI, typename TO, int OP, bool IMM>
int launch_typed1_k(const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const int64_t per_block = (int64_t)THREADS * typed1_u<TI, (OP == TADMA_OP_COPY || IMM) ? 1 : 2>();
    const int64_t want = (nvec + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    if (p.rank == 1) (void)launch_pdl(typed1_kernel<TI, TO, OP, IMM, true>, dim3(grid), dim3(THREADS), 0, s, p);
    else (void)launch_pdl(typed1_kernel<TI, TO, OP, IMM, false>, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename TI, typename TO, bool IMM>
int launch_typed1_op(int op, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (op) {
    case TADMA_OP_ADD: return launch_typed1_k<TI, TO, TADMA_OP_ADD, IMM>(p, nvec, s);
    case TADMA_OP_SUB: return launch_typed1_k<TI, TO, TADMA_OP_SUB, IMM>(p, nvec, s);
    case TADMA_OP_MUL: return launch_typed1_k<TI, TO, TADMA_OP_MUL, IMM>(p, nvec, s);
    case TADMA_OP_DIV: return launch_typed1_k<TI, TO, TADMA_OP_DIV, IMM>(p, nvec, s);
    case TADMA_OP_RSUB: return launch_typed1_k<TI, TO, TADMA_OP_RSUB, IMM>(p, nvec, s);
    case TADMA_OP_RDIV: return launch_typed1_k<TI, TO, TADMA_OP_RDIV, IMM>(p, nvec, s);
    case TADMA_OP_MAX: return launch_typed1_k<TI, TO, TADMA_OP_MAX, IMM>(p, nvec, s);
    default: return launch_typed1_k<TI, TO, TADMA_OP_MIN, IMM>(p, nvec, s);
    }
}

// Binary ops with an immediate or a second operand; casts / copies for every
// (TI, TO) pair.  Same-dtype binary ops only (TI == TO), the eager API's case.
template <typename TI, typename TO>
int launch_typed1_io(int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    if (op == TADMA_OP_COPY) return launch_typed1_k<TI, TO, TADMA_OP_COPY, false>(p, nvec, s);
    if constexpr (std::is_same<TI, TO>::value) {
        return imm ? launch_typed1_op<TI, TO, true>(op, p, nvec, s) : launch_typed1_op<TI, TO, false>(op, p, nvec, s);
    }
    return TADMA_ERR_UNSUPPORTED;
}

template <typename TI>
int launch_typed1_i(int odt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (odt) {
    case TADMA_F32: return launch_typed1_io<TI, float>(op, imm, p, nvec, s);
    case TADMA_F16: return launch_typed1_io<TI, __half>(op, imm, p, nvec, s);
    default: return launch_typed1_io<TI, __nv_bfloat16>(op, imm, p, nvec, s);
    }
}

int launch_typed1(int idt, int odt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (idt) {
    case TADMA_F32: return launch_typed1_i<float>(odt, op, imm, p, nvec, s);
    case TADMA_F16: return launch_typed1_i<__half>(odt, op, imm, p, nvec, s);
    default: return launch_typed1_i<__nv_bfloat16>(odt, op, imm, p, nvec, s);
    }
}

// Comparisons of one float dtype (a tensor or an immediate on the right) into
// a bool tensor, and where(bool or u8 condition, T, T) -> T: the mask
// producers and consumers of generated graphs, typed like typed1_kernel.
__device__ __forceinline__ void store_bytes8(uint8_t* p, const float (&v)[V]) {
    uint2 w = make_uint2(0u, 0u);
#pragma unroll
    for (int j = 0; j < V; j++) {
        const uint32_t b = (v[j] != 0.0f ? 1u : 0u) << (8 * (j & 3));
        if (j < 4) w.x |= b;
        else w.y |= b;
    }
    __stcs(reinterpret_cast<uint2*>(p), w);
}

template <typename TI, int OP, bool IMM, bool R1>
__global__ void __launch_bounds__(THREADS) typed_cmp_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int U = 2;
    constexpr int NIN = IMM ? 1 : 2;
    const float imm = __double2float_rn(p.prog[0].imm);
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        Raw8x<TI> raw[U][NIN];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NIN];
                typed_offsets<NIN, R1>(p, vi, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    raw8_load<TI>(reinterpret_cast<const TI*>(p.in[k].base) + io[k], raw[u][k], p.in[k].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                float a[V], b[V];
                raw8_cvt<TI>(raw[u][0], a);
                if constexpr (!IMM) raw8_cvt<TI>(raw[u][1], b);
#pragma unroll
                for (int j = 0; j < V; j++) a[j] = binary(OP, a[j], IMM ? imm : b[j], 0.0f);
                store_bytes8(reinterpret_cast<uint8_t*>(p.out) + oo[u], a);
            }
        }
    }
}

template <typename T, bool R1>
__global__ void __launch_bounds__(THREADS) typed_where_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int U = 2;
    const bool cond_bool = p.in[0].dtype == TADMA_BOOL;
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        uint2 c[U];
        Raw8x<T> x[U], y[U];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[3];
                typed_offsets<3, R1>(p, vi, oo[u], io);
                const uint8_t* cp = reinterpret_cast<const uint8_t*>(p.in[0].base) + io[0];
                c[u] = p.in[0].streaming ? __ldcs(reinterpret_cast<const uint2*>(cp)) : *reinterpret_cast<const uint2*>(cp);
                raw8_load<T>(reinterpret_cast<const T*>(p.in[1].base) + io[1], x[u], p.in[1].streaming);
                raw8_load<T>(reinterpret_cast<const T*>(p.in[2].base) + io[2], y[u], p.in[2].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                float fx[V], fy[V];
                raw8_cvt<T>(x[u], fx);
                raw8_cvt<T>(y[u], fy);
#pragma unroll
                for (int j = 0; j < V; j++) {
                    const uint32_t byte = ((j < 4 ? c[u].x : c[u].y) >> (8 * (j & 3))) & 0xffu;
                    const float cv = cond_bool ? (byte != 0u ? 1.0f : 0.0f) : (float)byte;
                    fx[j] = binary(TADMA_OP_WHERE, cv, fx[j], fy[j]);
                }
                raw8_store<T>(reinterpret_cast<T*>(p.out) + oo[u], fx);
            }
        }
    }
}

template <typename K>
int launch_grid2(K kernel, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const int64_t per_block = (int64_t)THREADS * 2;
    const int64_t want = (nvec + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    (void)launch_pdl(kernel, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename TI, int OP, bool IMM>
int launch_cmp_k(const ChainParams& p, int64_t nvec, cudaStream_t s) {
    return p.rank == 1 ? launch_grid2(typed_cmp_kernel<TI, OP, IMM, true>, p, nvec, s)
                       : launch_grid2(typed_cmp_kernel<TI, OP, IMM, false>, p, nvec, s);
}
template <typename TI, bool IMM>
int launch_cmp_op(int op, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (op) {
    case TADMA_OP_EQ: return launch_cmp_k<TI, TADMA_OP_EQ, IMM>(p, nvec, s);
    case TADMA_OP_NE: return launch_cmp_k<TI, TADMA_OP_NE, IMM>(p, nvec, s);
    case TADMA_OP_LT: return launch_cmp_k<TI, TADMA_OP_LT, IMM>(p, nvec, s);
    case TADMA_OP_GT: return launch_cmp_k<TI, TADMA_OP_GT, IMM>(p, nvec, s);
    case TADMA_OP_LE: return launch_cmp_k<TI, TADMA_OP_LE, IMM>(p, nvec, s);
    default: return launch_cmp_k<TI, TADMA_OP_GE, IMM>(p, nvec, s);
    }
}
// idt in {F32, F16, BF16}; the output is a bool tensor.
int launch_cmp(int idt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (idt) {
    case TADMA_F32: return imm ? launch_cmp_op<float, true>(op, p, nvec, s) : launch_cmp_op<float, false>(op, p, nvec, s);
    case TADMA_F16: return imm ? launch_cmp_op<__half, true>(op, p, nvec, s) : launch_cmp_op<__half, false>(op, p, nvec, s);
    default:
        return imm ? launch_cmp_op<__nv_bfloat16, true>(op, p, nvec, s) : launch_cmp_op<__nv_bfloat16, false>(op, p, nvec, s);
    }
}
// dt in {F32, F16, BF16}: the branches' and the output's dtype.
int launch_where(int dt, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const bool r1 = p.rank == 1;
    switch (dt) {
    case TADMA_F32: return r1 ? launch_grid2(typed_where_kernel<float, true>, p, nvec, s)
                              : launch_grid2(typed_where_kernel<float, false>, p, nvec, s);
    case TADMA_F16: return r1 ? launch_grid2(typed_where_kernel<__half, true>, p, nvec, s)
                              : launch_grid2(typed_where_kernel<__half, false>, p, nvec, s);
    default: return r1 ? launch_grid2(typed_where_kernel<__nv_bfloat16, true>, p, nvec, s)
                       : launch_grid2(typed_where_kernel<__nv_bfloat16, false>, p, nvec, s);
    }
}

template <typename TI, typename TO, int NIN, bool FAST>
int launch_typed_k(const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const int64_t per_block = (int64_t)THREADS * typed_steps<TI>();
    const int64_t want = (nvec + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    if (p.rank == 1) (void)launch_pdl(typed_kernel<TI, TO, NIN, FAST, true>, dim3(grid), dim3(THREADS), 0, s, p);
    else (void)launch_pdl(typed_kernel<TI, TO, NIN, FAST, false>, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename TI, typename TO>
int launch_typed_io(int nin, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    if constexpr (sizeof(TO) == 2) {
        if (fast) return nin == 1 ? launch_typed_k<TI, TO, 1, true>(p, nvec, s) : launch_typed_k<TI, TO, 2, true>(p, nvec, s);
    }
    return nin == 1 ? launch_typed_k<TI, TO, 1, false>(p, nvec, s) : launch_typed_k<TI, TO, 2, false>(p, nvec, s);
}

template <typename TI>
int launch_typed_i(int odt, int nin, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (odt) {
    case TADMA_F32: return launch_typed_io<TI, float>(nin, fast, p, nvec, s);
    case TADMA_F16: return launch_typed_io<TI, __half>(nin, fast, p, nvec, s);
    default: return launch_typed_io<TI, __nv_bfloat16>(nin, fast, p, nvec, s);
    }
}

// idt, odt in {F32, F16, BF16}; nin in {1, 2}.
int launch_typed(int idt, int odt, int nin, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (idt) {
    case TADMA_F32: return launch_typed_i<float>(odt, nin, fast, p, nvec, s);
    case TADMA_F16: return launch_typed_i<__half>(odt, nin, fast, p, nvec, s);
    default: return launch_typed_i<__nv_bfloat16>(odt, nin, fast, p, nvec, s);
    }
}

// ---------------------------------------------------------- tiled transpose --
//
// One input whose unit-stride dim is not the output's: a copy through a
// transpose (contiguous() after transpose<0,2,3,1>, a cast of a transposed
// view).  Element-at-a-time, one side of the copy would be uncoalesced; here
// a CTA stages a 32 x 32 tile in shared memory, reading along the input's
// contiguous dim and writing along the output's, and runs the chain on each
// element on the way out.  Remaining dims are batch dims (grid z).

struct TransposeParams {
    const char* in;
    char* out;
    int32_t in_dtype, out_dtype;
    int64_t n_i, n_j;    // i: the input's unit-stride dim; j: the output's
    int64_t in_sj;       // input stride along j
    int64_t out_si;      // output stride along i
    int32_t nb, pad;     // batch dims
    int64_t nbatch;
    DivMod bdm[TADMA_MAX_RANK];
    int64_t b_in[TADMA_MAX_RANK], b_out[TADMA_MAX_RANK];
    ChainParams chain;   // the program (n_instr, prog, scale)
};

template <int PROG>
__global__ void __launch_bounds__(THREADS) transpose_chain_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    __shared__ float tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
    const int64_t i0 = (int64_t)blockIdx.y * 32, j0 = (int64_t)blockIdx.x * 32;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t q, r;
            tp.bdm[d].divmod(e, q, r);
            ib += (int64_t)r * tp.b_in[d];
            ob += (int64_t)r * tp.b_out[d];
            e = q;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t i = i0 + tx, j = j0 + ty + 8 * k;
            if (i < tp.n_i && j < tp.n_j) tile[ty + 8 * k][tx] = load_as<float>(tp.in, tp.in_dtype, ib + i + j * tp.in_sj);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t i = i0 + ty + 8 * k, j = j0 + tx;
            if (i < tp.n_i && j < tp.n_j) {
                float val[1][1] = {{tile[tx][ty + 8 * k]}};
                float acc[1] = {val[0][0]};
                program<float, 1, 1, PROG>(tp.chain, acc, val);
                store_from(tp.out, tp.out_dtype, ob + i * tp.out_si + j, acc[0]);
            }
        }
        __syncthreads();
    }
}

// 64 x 64 tiles with 16-byte accesses on both sides, for f32 / f16 / bf16 in
// and out with 16-byte aligned rows and fp32 on at least one side (16-bit in
// and out goes to transpose16_kernel): each thread loads 2 (16-bit) or 4 (f32)
// 16-byte vectors along the input's contiguous dim, the tile is transposed
// through shared memory as fp32, and each thread stores 2 vectors of 8
// elements along the output's contiguous dim.  One tile per CTA.  The 32 x 32
// element-at-a-time kernel above (the fallback for other layouts) kept too
// few bytes in flight: ~1.0 TB/s for a 16-bit transpose.
template <typename TI, typename TO, int PROG>
__global__ void __launch_bounds__(THREADS) transpose64_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    constexpr int T = 64;
    constexpr int VI = 16 / (int)sizeof(TI);        // input elements per 16-byte load
    constexpr int LV = T * (T / VI) / THREADS;       // loads per thread
    constexpr int SV = T * (T / 8) / THREADS;        // 8-element stores per thread
    __shared__ float tile[T][T + 1];                 // [j][i]
    const int64_t i0 = (int64_t)blockIdx.y * T, j0 = (int64_t)blockIdx.x * T;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t q, r;
            tp.bdm[d].divmod(e, q, r);
            ib += (int64_t)r * tp.b_in[d];
            ob += (int64_t)r * tp.b_out[d];
            e = q;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
        const TI* in = reinterpret_cast<const TI*>(tp.in) + ib;
        uint4 r[LV];
#pragma unroll
        for (int u = 0; u < LV; u++) {
            const int q = threadIdx.x + THREADS * u;
            const int jj = q / (T / VI), ii = (q % (T / VI)) * VI;
            const int64_t i = i0 + ii, j = j0 + jj;
            if (i < tp.n_i && j < tp.n_j) r[u] = ld_stream_v4(in + i + j * tp.in_sj);
        }
#pragma unroll
        for (int u = 0; u < LV; u++) {
            const int q = threadIdx.x + THREADS * u;
            const int jj = q / (T / VI), ii = (q % (T / VI)) * VI;
            if (i0 + ii < tp.n_i && j0 + jj < tp.n_j) {
                float f[8];
                if constexpr (sizeof(TI) == 4) {
                    f[0] = __uint_as_float(r[u].x);
                    f[1] = __uint_as_float(r[u].y);
                    f[2] = __uint_as_float(r[u].z);
                    f[3] = __uint_as_float(r[u].w);
                } else {
                    unpack8(r[u], std::is_same<TI, __half>::value ? TADMA_F16 : TADMA_BF16, f);
                }
#pragma unroll
                for (int k = 0; k < VI; k++) tile[jj][ii + k] = f[k];
            }
        }
        __syncthreads();
        TO* out = reinterpret_cast<TO*>(tp.out) + ob;
#pragma unroll
        for (int u = 0; u < SV; u++) {
            const int q = threadIdx.x + THREADS * u;
            const int ii = q >> 3, jj = (q & 7) * 8;
            const int64_t i = i0 + ii, j = j0 + jj;
            if (i < tp.n_i && j < tp.n_j) {
                float val[1][8], acc[8];
#pragma unroll
                for (int k = 0; k < 8; k++) acc[k] = val[0][k] = tile[jj + k][ii];
                program<float, 1, 8, PROG>(tp.chain, acc, val);
                raw8_store<TO>(out + i * tp.out_si + j, acc);
            }
        }
        __syncthreads();
    }
}

// 16-bit in and out: 64 (i) x TJ (j) tiles kept as 16-bit element pairs.
// Each thread loads the same 16-byte chunk (8 values of i) from two adjacent
// input rows j, j + 1 and packs value k of both into one 32-bit word: the
// output row i + k's elements j, j + 1.  Words go to shared memory as
// W[i][j / 2]; the output side reads 16-byte chunks of 4 words (8 values of
// j) and stores them along the output's contiguous dim.  The 4-word chunks of
// row i are swizzled by XOR with (i / 8) % 8, so the scalar word stores (8
// rows i = 8c + k, c = 0..7, per warp) and the 16-byte reads (8 consecutive
// chunks per quarter warp) each cover all 32 banks once.  Half the shared
// memory traffic of an fp32 tile, and TJ = 256 keeps 32 KB of loads in flight
// per CTA (4x the 64 x 64 tile).  RAW: the chain is an identity on the same
// dtype, so words are stored untouched (bit-exact, NaN payloads included).
template <typename TI, typename TO, int PROG, int TJ, bool RAW>
__global__ void __launch_bounds__(THREADS, 4) transpose16_kernel(const __grid_constant__ TransposeParams tp) {
    pdl_begin();
    static_assert(sizeof(TI) == 2 && sizeof(TO) == 2 && (TJ == 128 || TJ == 256));
    constexpr int TI_ = 64;
    constexpr int WPR = TJ / 2;                  // words per W row
    constexpr int NP = TJ / 64;                  // row pairs per thread (32 pairs per pass)
    constexpr int CPR = TJ / 8;                  // 16-byte output chunks per W row
    constexpr int RPP = THREADS / CPR;           // W rows per output pass
    constexpr int NS = TI_ / RPP;                // output chunks per thread
    __shared__ __align__(16) uint32_t W[TI_ * WPR];
    const int t = threadIdx.x;
    const int c = t & 7, p0 = t >> 3;            // input chunk (i = 8c..8c+7), first row pair
    const int q = t % CPR, r0 = t / CPR;         // output chunk (j = 8q..8q+7), first W row
    const int64_t i0 = (int64_t)blockIdx.y * TI_, j0 = (int64_t)blockIdx.x * TJ;
    for (int64_t bz = blockIdx.z; bz < tp.nbatch; bz += gridDim.z) {
        uint64_t e = (uint64_t)bz;
        int64_t ib = 0, ob = 0;
        for (int d = tp.nb - 1; d >= 1; d--) {
            uint64_t qq, rr;
            tp.bdm[d].divmod(e, qq, rr);
            ib += (int64_t)rr * tp.b_in[d];
            ob += (int64_t)rr * tp.b_out[d];
            e = qq;
        }
        if (tp.nb > 0) {
            ib += (int64_t)e * tp.b_in[0];
            ob += (int64_t)e * tp.b_out[0];
        }
        const TI* in = reinterpret_cast<const TI*>(tp.in) + ib;
        const int64_t i = i0 + 8 * c;
        uint4 a[NP], b[NP];
#pragma unroll
        for (int u = 0; u < NP; u++) {
            const int64_t j = j0 + 2 * (p0 + 32 * u);
            // n_j is a multiple of 8, so j < n_j implies j + 1 < n_j.
            if (i < tp.n_i && j < tp.n_j) {
                a[u] = ld_stream_v4(in + i + j * tp.in_sj);
                b[u] = ld_stream_v4(in + i + (j + 1) * tp.in_sj);
            } else {
                a[u] = b[u] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < NP; u++) {
            const int p = p0 + 32 * u;
            const int pw = (((p >> 2) ^ c) << 2) | (p & 3);  // swizzled word of row 8c + k
            const uint32_t av[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
            const uint32_t bv[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
#pragma unroll
            for (int h = 0; h < 4; h++) {
                W[(8 * c + 2 * h) * WPR + pw] = __byte_perm(av[h], bv[h], 0x5410);
                W[(8 * c + 2 * h + 1) * WPR + pw] = __byte_perm(av[h], bv[h], 0x7632);
            }
        }
        __syncthreads();
        TO* out = reinterpret_cast<TO*>(tp.out) + ob;
#pragma unroll
        for (int u = 0; u < NS; u++) {
            const int row = r0 + RPP * u;
            const int64_t oi = i0 + row, oj = j0 + 8 * q;
            if (oi < tp.n_i && oj < tp.n_j) {
                const uint4 w = *reinterpret_cast<const uint4*>(&W[row * WPR + ((q ^ ((row >> 3) & 7)) << 2)]);
                if constexpr (RAW) {
                    st_stream_v4(out + oi * tp.out_si + oj, w);
                } else {
                    float val[1][8], acc[8];
                    unpack8(w, std::is_same<TI, __half>::value ? TADMA_F16 : TADMA_BF16, val[0]);
#pragma unroll
                    for (int k = 0; k < 8; k++) acc[k] = val[0][k];
                    program<float, 1, 8, PROG>(tp.chain, acc, val);
                    raw8_store<TO>(out + oi * tp.out_si + oj, acc);
                }
            }
        }
        __syncthreads();
    }
}

template <typename TI, typename TO>
void launch_t64_io(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    if (fast && sizeof(TO) == 2) (void)launch_pdl(transpose64_kernel<TI, TO, PROG_INTERP_FAST>, grid, dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose64_kernel<TI, TO, PROG_INTERP>, grid, dim3(THREADS), 0, s, tp);
}
template <typename TI>
void launch_t64_i(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    switch (tp.out_dtype) {
    case TADMA_F32: launch_t64_io<TI, float>(fast, grid, tp, s); break;
    case TADMA_F16: launch_t64_io<TI, __half>(fast, grid, tp, s); break;
    default: launch_t64_io<TI, __nv_bfloat16>(fast, grid, tp, s); break;
    }
}

// Whether transpose64_kernel covers this layout: f32 / f16 / bf16 on both
// sides, every row start and batch offset 16-byte aligned, and whole vectors
// at the edges (n_i a multiple of the input vector, n_j of 8).
bool transpose64_ok(const TransposeParams& tp) {
    auto fdt = [](int dt) { return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16; };
    if (!fdt(tp.in_dtype) || !fdt(tp.out_dtype)) return false;
    const int64_t ei = dtype_size(tp.in_dtype), eo = dtype_size(tp.out_dtype);
    if ((uintptr_t)tp.in % 16 || (uintptr_t)tp.out % 16) return false;
    if ((tp.in_sj * ei) % 16 || (tp.out_si * eo) % 16) return false;
    for (int d = 0; d < tp.nb; d++)
        if ((tp.b_in[d] * ei) % 16 || (tp.b_out[d] * eo) % 16) return false;
    if (tp.n_i % (16 / ei) || tp.n_j % 8) return false;
    return (tp.n_i + 63) / 64 <= 65535;
}

// ------------------------------------------------------------ host side --

// ------------------------------------------------------ chain reduction --
//
// tadma_b200_reduce_chain: a reduction whose elements are a fused chain of
// up to 4 broadcast operands, evaluated on the fly.  One warp per output
// element (the kept dims, folded); its lanes walk the reduced axis.  With the
// axis contiguous (stride 1) or broadcast (stride 0) in every operand and
// fp32 compute, lanes take 8 elements per step with 16-byte loads (the
// eltwise vector loader) and run the chain on the 8 at once; otherwise one
// element per lane step.  Lanes fold their elements in increasing index
// order and combine in a fixed butterfly, as the reduction kernels do.

// Raw 16-byte words of one 8-element vector (fp32: 2 words, fp16 / bf16: 1),
// converted to the compute type at use.
struct RawV {
    uint4 a, b;
};
__device__ __forceinline__ void load_raw_vec(const Operand& o, int64_t off, RawV& r) {
    const char* p = o.base + off * dtype_size(o.dtype);
    r.a = ld_stream_v4(p);
    if (o.dtype == TADMA_F32) r.b = ld_stream_v4(p + 16);
}
template <typename C>
__device__ __forceinline__ void cvt_raw_vec(int dt, const RawV& r, C (&v)[V]) {
    if (dt == TADMA_F32) {
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = from_f<C>(__uint_as_float(w[j]));
    } else {
        float f[8];
        unpack8(r.a, dt, f);
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = from_f<C>(f[j]);
    }
}

struct ChainReduceParams {
    ChainParams chain;  // prog, n_instr and the operands (base, dtype, inner_bcast)
    int32_t n_ins, square, post, out_dtype;
    int64_t R;                        // reduced extent
    int64_t ax[TADMA_MAX_INPUTS];     // operand strides along the reduced axis
    int64_t nrows;                    // output elements
    int32_t krank, pad;
    DivMod kdm[TADMA_MAX_RANK];
    int64_t kin[TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    int64_t kout[TADMA_MAX_RANK];
    char* out;
};

constexpr int POST_NONE = 0, POST_MEAN = 1, POST_RMS = 2;

template <typename C, int K, bool VEC, int NIN>
__global__ void __launch_bounds__(THREADS, !VEC ? 2 : NIN == 1 ? 3 : 2) chain_reduce_kernel(const __grid_constant__ ChainReduceParams p) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    for (int64_t row = gw; row < p.nrows; row += nw) {
        int64_t base[TADMA_MAX_INPUTS] = {0, 0, 0, 0};
        int64_t ooff = 0;
        {
            uint64_t e = (uint64_t)row;
            for (int d = p.krank - 1; d >= 0; d--) {
                uint64_t q, r;
                if (d > 0) {
                    p.kdm[d].divmod(e, q, r);
                } else {
                    r = e;
                    q = 0;
                }
                ooff += (int64_t)r * p.kout[d];
#pragma unroll
                for (int k = 0; k < TADMA_MAX_INPUTS; k++) base[k] += (int64_t)r * p.kin[k][d];
                e = q;
            }
        }
        State<C> s = init_state<K, C>();
        int64_t done = 0;
        if constexpr (VEC) {
            // An operand broadcast along the axis is one value per output,
            // loaded once.  The others are double-buffered as raw 16-byte
            // words: the next vector step's loads are in flight while this
            // step converts, runs the chain and folds.
            const int64_t nv = p.R / V;
            C bc[NIN];
#pragma unroll
            for (int k = 0; k < NIN; k++)
                bc[k] = p.ax[k] == 0 ? load_as<C>(p.chain.in[k].base, p.chain.in[k].dtype, base[k]) : C(0);
            RawV cur[NIN], nxt[NIN];
            int64_t v = lane;
            if (v < nv) {
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    if (p.ax[k] != 0) load_raw_vec(p.chain.in[k], base[k] + v * V, cur[k]);
            }
            for (; v < nv; v += 32) {
                if (v + 32 < nv) {
#pragma unroll
                    for (int k = 0; k < NIN; k++)
                        if (p.ax[k] != 0) load_raw_vec(p.chain.in[k], base[k] + (v + 32) * V, nxt[k]);
                }
                C val[NIN][V];
#pragma unroll
                for (int k = 0; k < NIN; k++) {
                    if (p.ax[k] == 0) {
#pragma unroll
                        for (int j = 0; j < V; j++) val[k][j] = bc[k];
                    } else {
                        cvt_raw_vec<C>(p.chain.in[k].dtype, cur[k], val[k]);
                    }
                }
                C acc[V];
#pragma unroll
                for (int j = 0; j < V; j++) acc[j] = val[0][j];
                run_chain<C, NIN, V, false>(p.chain, acc, val);
#pragma unroll
                for (int j = 0; j < V; j++) update<K, C>(s, p.square ? acc[j] * acc[j] : acc[j], v * V + j);
#pragma unroll
                for (int k = 0; k < NIN; k++) cur[k] = nxt[k];
            }
            done = nv * V;
        }
        for (int64_t r = done + lane; r < p.R; r += 32) {
            C val[TADMA_MAX_INPUTS][1];
#pragma unroll
            for (int k = 0; k < TADMA_MAX_INPUTS; k++)
                if (k < p.n_ins) val[k][0] = load_as<C>(p.chain.in[k].base, p.chain.in[k].dtype, base[k] + r * p.ax[k]);
            C acc[1] = {p.n_ins > 0 ? val[0][0] : C(0)};
            run_chain<C, TADMA_MAX_INPUTS, 1, false>(p.chain, acc, val);
            update<K, C>(s, p.square ? acc[0] * acc[0] : acc[0], r);
        }
        s = warp_combine<K, C>(s);
        if (lane == 0) {
            if constexpr (K == K_ARGMAX || K == K_ARGMIN) {
                store_from(p.out, p.out_dtype, ooff, (int64_t)(s.i < 0 ? 0 : s.i));
            } else {
                C v = s.v;
                if constexpr (std::is_floating_point<C>::value) {
                    if (p.post == POST_MEAN) v = v / (C)p.R;
                    else if (p.post == POST_RMS) v = sqrt(v / (C)p.R);
                } else {
                    if (p.post == POST_MEAN) v = v / p.R;
                }
                store_from(p.out, p.out_dtype, ooff, v);
            }
        }
    }
}

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

// `narrow`: fp32 compute and every operand narrow (see load_raw_narrow).
template <typename C, int NIN, int PROG>
int launch(const ChainParams& p, bool vec, int64_t work, cudaStream_t s, bool narrow = false) {
    narrow = narrow && vec && std::is_same<C, float>::value;
    const int64_t per_block = (int64_t)THREADS * (!vec ? SU : narrow ? narrow_steps<NIN>() : vec_steps<NIN>());
    const int64_t want = (work + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    if (narrow) {
        if constexpr (std::is_same<C, float>::value)
            (void)launch_pdl(chain_narrow_kernel<NIN, PROG>, dim3(grid), dim3(THREADS), 0, s, p);
    } else if (vec) {
        (void)launch_pdl(chain_vec_kernel<C, NIN, PROG>, dim3(grid), dim3(THREADS), 0, s, p);
    } else {
        (void)launch_pdl(chain_scalar_kernel<C, NIN, PROG>, dim3(grid), dim3(THREADS), 0, s, p);
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

// Interpreter launch; `fast` and `narrow` only exist for fp32 compute.
template <typename C>
int launch_interp(int nin, bool fast, const ChainParams& p, bool vec, int64_t work, cudaStream_t s, bool narrow) {
    if constexpr (std::is_same<C, float>::value) {
        if (fast) {
            switch (nin) {
            case 0: return launch<C, 0, PROG_INTERP_FAST>(p, vec, work, s, narrow);
            case 1: return launch<C, 1, PROG_INTERP_FAST>(p, vec, work, s, narrow);
            case 2: return launch<C, 2, PROG_INTERP_FAST>(p, vec, work, s, narrow);
            case 3: return launch<C, 3, PROG_INTERP_FAST>(p, vec, work, s, narrow);
            default: return launch<C, 4, PROG_INTERP_FAST>(p, vec, work, s, narrow);
            }
        }
    }
    switch (nin) {
    case 0: return launch<C, 0, PROG_INTERP>(p, vec, work, s, narrow);
    case 1: return launch<C, 1, PROG_INTERP>(p, vec, work, s, narrow);
    case 2: return launch<C, 2, PROG_INTERP>(p, vec, work, s, narrow);
    case 3: return launch<C, 3, PROG_INTERP>(p, vec, work, s, narrow);
    default: return launch<C, 4, PROG_INTERP>(p, vec, work, s, narrow);
    }
}

// Affine + activation vector kernels (fp32 compute).
template <int ACT, bool FAST, bool MUL>
int launch_affine_add(bool add, const ChainParams& p, int64_t work, cudaStream_t s, bool narrow) {
    if (add) return launch<float, 2, affine_prog(ACT, FAST, MUL, true)>(p, true, work, s, narrow);
    return launch<float, 1, affine_prog(ACT, FAST, MUL, false)>(p, true, work, s, narrow);
}
template <int ACT, bool FAST>
int launch_affine_mul(bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s, bool narrow) {
    return mul ? launch_affine_add<ACT, FAST, true>(add, p, work, s, narrow)
               : launch_affine_add<ACT, FAST, false>(add, p, work, s, narrow);
}
template <int ACT>
int launch_affine_fast(bool fast, bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s, bool narrow) {
    return fast ? launch_affine_mul<ACT, true>(mul, add, p, work, s, narrow)
                : launch_affine_mul<ACT, false>(mul, add, p, work, s, narrow);
}
int launch_affine(int act, bool fast, bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s,
                  bool narrow) {
    switch (act) {
    case ACT_GELU: return launch_affine_fast<ACT_GELU>(fast, mul, add, p, work, s, narrow);
    case ACT_RELU: return launch_affine_fast<ACT_RELU>(fast, mul, add, p, work, s, narrow);
    case ACT_SIGMOID: return launch_affine_fast<ACT_SIGMOID>(fast, mul, add, p, work, s, narrow);
    case ACT_TANH: return launch_affine_fast<ACT_TANH>(fast, mul, add, p, work, s, narrow);
    default: return launch_affine_fast<ACT_NONE>(fast, mul, add, p, work, s, narrow);
    }
}

// Recognises [MUL imm]? [ADD ins[1]]? [GELU | RELU | SIGMOID | TANH]? in fp32
// compute with only no-op roundings (fp32 / fp64): act(x * s + b).
struct AffineMatch {
    bool ok = false, mul = false, add = false;
    int act = ACT_NONE;
    float scale = 1.0f;
};

AffineMatch match_affine(const tadma_instr* prog, int n_instr, int n_ins) {
    AffineMatch m;
    auto noop_round = [](int rd) { return rd < 0 || rd == TADMA_F32 || rd == TADMA_F64; };
    int i = 0;
    if (i < n_instr && prog[i].op == TADMA_OP_MUL && prog[i].b == TADMA_SRC_IMM && noop_round(prog[i].round_dtype)) {
        m.mul = true;
        m.scale = (float)prog[i].imm;
        i++;
    }
    if (i < n_instr && prog[i].op == TADMA_OP_ADD && prog[i].b == 1 && noop_round(prog[i].round_dtype)) {
        m.add = true;
        i++;
    }
    if (i < n_instr && noop_round(prog[i].round_dtype)) {
        switch (prog[i].op) {
        case TADMA_OP_GELU: m.act = ACT_GELU; i++; break;
        case TADMA_OP_RELU: m.act = ACT_RELU; i++; break;
        case TADMA_OP_SIGMOID: m.act = ACT_SIGMOID; i++; break;
        case TADMA_OP_TANH: m.act = ACT_TANH; i++; break;
        default: break;
        }
    }
    m.ok = i == n_instr && n_instr > 0 && n_ins == (m.add ? 2 : 1);
    return m;
}

template <typename XT, typename OT, int ACT>
int launch_rows_t(const AffineRowsParams& p, cudaStream_t s) {
    const int64_t ncb = (p.ncv + THREADS - 1) / THREADS;
    const int64_t tiles = (p.rows + affine_rb<XT>() - 1) / affine_rb<XT>();
    if (ncb * tiles > 0x7fffffff) return fail(TADMA_ERR_UNSUPPORTED, "eltwise: more than 2^31 row tiles");
    cudaError_t e = launch_pdl(affine_rows_kernel<XT, OT, ACT>, dim3((unsigned)(ncb * tiles)), dim3(THREADS), 0, s, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename XT, typename OT>
int launch_rows_act(int act, const AffineRowsParams& p, cudaStream_t s) {
    switch (act) {
    case ACT_GELU: return launch_rows_t<XT, OT, ACT_GELU>(p, s);
    case ACT_RELU: return launch_rows_t<XT, OT, ACT_RELU>(p, s);
    case ACT_SIGMOID: return launch_rows_t<XT, OT, ACT_SIGMOID>(p, s);
    case ACT_TANH: return launch_rows_t<XT, OT, ACT_TANH>(p, s);
    default: return launch_rows_t<XT, OT, ACT_NONE>(p, s);
    }
}

// x dtype = bias dtype in {f32, f16, bf16}; out dtype = x dtype or f32.
int launch_rows(int xdt, int odt, int act, const AffineRowsParams& p, cudaStream_t s) {
    if (xdt == TADMA_F32) return launch_rows_act<float, float>(act, p, s);
    if (xdt == TADMA_F16)
        return odt == TADMA_F16 ? launch_rows_act<__half, __half>(act, p, s) : launch_rows_act<__half, float>(act, p, s);
    return odt == TADMA_BF16 ? launch_rows_act<__nv_bfloat16, __nv_bfloat16>(act, p, s)
                             : launch_rows_act<__nv_bfloat16, float>(act, p, s);
}

// Whether the chain leaves a value of the input dtype unchanged: only copies
// of the running value, rounded (if at all) to the input dtype or wider.
bool identity_chain(const TransposeParams& tp) {
    if (tp.in_dtype != tp.out_dtype) return false;
    for (int k = 0; k < tp.chain.n_instr; k++) {
        const tadma_instr& I = tp.chain.prog[k];
        if (I.op != TADMA_OP_COPY || I.b == TADMA_SRC_IMM) return false;
        const int rd = I.round_dtype;
        if (rd >= 0 && rd != tp.in_dtype && rd != TADMA_F32 && rd != TADMA_F64) return false;
    }
    return true;
}

template <typename TI, typename TO, int TJ>
void launch_t16_tj(bool fast, dim3 grid, const TransposeParams& tp, cudaStream_t s) {
    if (identity_chain(tp)) (void)launch_pdl(transpose16_kernel<TI, TO, PROG_INTERP, TJ, true>, grid, dim3(THREADS), 0, s, tp);
    else if (fast) (void)launch_pdl(transpose16_kernel<TI, TO, PROG_INTERP_FAST, TJ, false>, grid, dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose16_kernel<TI, TO, PROG_INTERP, TJ, false>, grid, dim3(THREADS), 0, s, tp);
}
template <typename TI, typename TO>
void launch_t16_io(bool fast, int64_t gz, const TransposeParams& tp, cudaStream_t s) {
    const unsigned gy = (unsigned)((tp.n_i + 63) / 64);
    if (tp.n_j >= 256) launch_t16_tj<TI, TO, 256>(fast, dim3((unsigned)((tp.n_j + 255) / 256), gy, (unsigned)gz), tp, s);
    else launch_t16_tj<TI, TO, 128>(fast, dim3((unsigned)((tp.n_j + 127) / 128), gy, (unsigned)gz), tp, s);
}
template <typename TI>
void launch_t16_i(bool fast, int64_t gz, const TransposeParams& tp, cudaStream_t s) {
    if (tp.out_dtype == TADMA_F16) launch_t16_io<TI, __half>(fast, gz, tp, s);
    else launch_t16_io<TI, __nv_bfloat16>(fast, gz, tp, s);
}

int launch_transpose(bool fast, const TransposeParams& tp, cudaStream_t s) {
    const int64_t gz = tp.nbatch < 65535 ? tp.nbatch : 65535;
    const bool in16 = tp.in_dtype == TADMA_F16 || tp.in_dtype == TADMA_BF16;
    const bool out16 = tp.out_dtype == TADMA_F16 || tp.out_dtype == TADMA_BF16;
    if (in16 && out16 && transpose64_ok(tp)) {
        if (tp.in_dtype == TADMA_F16) launch_t16_i<__half>(fast, gz > 0 ? gz : 1, tp, s);
        else launch_t16_i<__nv_bfloat16>(fast, gz > 0 ? gz : 1, tp, s);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
    }
    if (transpose64_ok(tp)) {
        dim3 grid((unsigned)((tp.n_j + 63) / 64), (unsigned)((tp.n_i + 63) / 64), (unsigned)(gz > 0 ? gz : 1));
        switch (tp.in_dtype) {
        case TADMA_F32: launch_t64_i<float>(fast, grid, tp, s); break;
        case TADMA_F16: launch_t64_i<__half>(fast, grid, tp, s); break;
        default: launch_t64_i<__nv_bfloat16>(fast, grid, tp, s); break;
        }
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
    }
    const int64_t gx = (tp.n_j + 31) / 32, gy = (tp.n_i + 31) / 32;
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)(gz > 0 ? gz : 1));
    if (fast) (void)launch_pdl(transpose_chain_kernel<PROG_INTERP_FAST>, dim3(grid), dim3(THREADS), 0, s, tp);
    else (void)launch_pdl(transpose_chain_kernel<PROG_INTERP>, dim3(grid), dim3(THREADS), 0, s, tp);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

bool is_transcendental(int op) { return op >= TADMA_OP_EXP && op <= TADMA_OP_GELU && op != TADMA_OP_RELU; }

template <typename C, int K, bool VEC, int NIN>
int launch_chain_reduce_k(const ChainReduceParams& p, cudaStream_t s) {
    const void* fn = (const void*)chain_reduce_kernel<C, K, VEC, NIN>;
    const int64_t want = (p.nrows + (THREADS / 32) - 1) / (THREADS / 32);
    const int64_t cap = (int64_t)sm_count() * blocks_per_sm(fn);
    const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
    cudaError_t e = launch_pdl(chain_reduce_kernel<C, K, VEC, NIN>, dim3(grid), dim3(THREADS), 0, s, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_reduce_chain launch");
}

// The scalar path takes the operand count at run time (NIN = 4 arrays); the
// vector path is instantiated per operand count to keep its registers.
template <typename C, bool VEC, int NIN>
int launch_chain_reduce_n(int kind, const ChainReduceParams& p, cudaStream_t s) {
    switch (kind) {
    case K_SUM: return launch_chain_reduce_k<C, K_SUM, VEC, NIN>(p, s);
    case K_MAX: return launch_chain_reduce_k<C, K_MAX, VEC, NIN>(p, s);
    case K_MIN: return launch_chain_reduce_k<C, K_MIN, VEC, NIN>(p, s);
    case K_ARGMAX: return launch_chain_reduce_k<C, K_ARGMAX, VEC, NIN>(p, s);
    default: return launch_chain_reduce_k<C, K_ARGMIN, VEC, NIN>(p, s);
    }
}

template <typename C, bool VEC>
int launch_chain_reduce(int kind, const ChainReduceParams& p, cudaStream_t s) {
    if constexpr (!VEC) {
        return launch_chain_reduce_n<C, false, TADMA_MAX_INPUTS>(kind, p, s);
    } else {
        switch (p.n_ins) {
        case 1: return launch_chain_reduce_n<C, true, 1>(kind, p, s);
        case 2: return launch_chain_reduce_n<C, true, 2>(kind, p, s);
        case 3: return launch_chain_reduce_n<C, true, 3>(kind, p, s);
        default: return launch_chain_reduce_n<C, true, 4>(kind, p, s);
        }
    }
}

bool valid_op(int op) {
    return (op >= 0 && op <= TADMA_OP_NOT) || (op >= TADMA_OP_ADD && op <= TADMA_OP_LOR) || op == TADMA_OP_WHERE;
}

}  // namespace

// Same rule as the oracle: integer-only chains compute in int64, anything
// touching f64/i64 in f64, the rest in f32.
int resolve_compute(const tadma_tensor* out, const tadma_tensor* ins, int n_ins, const tadma_instr* prog, int n_instr,
                    int compute) {
    if (compute != TADMA_COMPUTE_AUTO) return compute;
    bool all_int = !dtype_is_float(out->dtype);
    bool any_wide = out->dtype == TADMA_F64 || out->dtype == TADMA_I64;
    for (int k = 0; k < n_ins; k++) {
        if (dtype_is_float(ins[k].dtype)) all_int = false;
        if (ins[k].dtype == TADMA_F64 || ins[k].dtype == TADMA_I64) any_wide = true;
    }
    for (int i = 0; i < n_instr; i++) {
        if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW) all_int = false;
        if ((prog[i].b == TADMA_SRC_IMM || prog[i].c == TADMA_SRC_IMM) && prog[i].imm != (double)(int64_t)prog[i].imm)
            all_int = false;
    }
    if (all_int) return TADMA_COMPUTE_I64;
    return any_wide ? TADMA_COMPUTE_F64 : TADMA_COMPUTE_F32;
}

}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_eltwise(const tadma_tensor* out, const tadma_tensor* ins, int32_t n_ins,
                                  const tadma_instr* prog, int32_t n_instr, int32_t compute, void* stream) {
    std::string err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (n_ins < 0 || n_ins > TADMA_MAX_INPUTS) return fail(TADMA_ERR_INVALID, "n_ins out of range [0, 4]");
    if (n_instr < 0 || n_instr > TADMA_MAX_INSTR) return fail(TADMA_ERR_INVALID, "n_instr out of range [0, 16]");
    if (n_ins > 0 && !ins) return fail(TADMA_ERR_INVALID, "ins is NULL");
    if (n_instr > 0 && !prog) return fail(TADMA_ERR_INVALID, "prog is NULL");
    for (int k = 0; k < n_ins; k++) {
        err = check_tensor(&ins[k], "ins[k]");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (ins[k].rank != out->rank) return fail(TADMA_ERR_INVALID, "ins[k] rank differs from out rank");
        for (int d = 0; d < out->rank; d++)
            if (ins[k].dims[d] != out->dims[d] && ins[k].dims[d] != 1)
                return fail(TADMA_ERR_INVALID, "ins[k] dims not broadcastable to out dims");
    }
    for (int i = 0; i < n_instr; i++) {
        const tadma_instr& I = prog[i];
        if (!valid_op(I.op)) return fail(TADMA_ERR_INVALID, "unknown op code");
        bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
        if (needs_b && !(I.b == TADMA_SRC_IMM || (I.b >= 0 && I.b < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector b out of range");
        if (I.op == TADMA_OP_WHERE && !(I.c == TADMA_SRC_IMM || (I.c >= 0 && I.c < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector c out of range");
        if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return fail(TADMA_ERR_INVALID, "bad round_dtype");
    }
    int cm = resolve_compute(out, ins, n_ins, prog, n_instr, compute);
    if (cm < TADMA_COMPUTE_F32 || cm > TADMA_COMPUTE_I64) return fail(TADMA_ERR_INVALID, "bad compute mode");
    if (cm == TADMA_COMPUTE_I64)
        for (int i = 0; i < n_instr; i++)
            if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW)
                return fail(TADMA_ERR_UNSUPPORTED, "transcendental op in int64 compute");
    const int64_t n = numel(out);
    if (n == 0) return TADMA_OK;

    // Joint fold of out + inputs.
    int64_t strides[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    for (int d = 0; d < out->rank; d++) {
        strides[0][d] = out->strides[d];
        for (int k = 0; k < n_ins; k++) strides[1 + k][d] = (ins[k].dims[d] == 1) ? 0 : ins[k].strides[d];
    }
    Folded f = fold(out->rank, out->dims, strides, 1 + n_ins);

    ChainParams p{};
    p.rank = f.rank;
    p.n_instr = n_instr;
    p.out_dtype = out->dtype;
    p.out = (char*)out->data;
    for (int d = 0; d < f.rank; d++) {
        p.dims[d] = f.dims[d];
        p.out_stride[d] = f.strides[0][d];
    }
    for (int k = 0; k < n_ins; k++) {
        Operand& o = p.in[k];
        o.base = (const char*)ins[k].data;
        o.dtype = ins[k].dtype;
        o.streaming = 1;
        for (int d = 0; d < f.rank; d++) {
            o.stride[d] = f.strides[1 + k][d];
            if (o.stride[d] == 0 && f.dims[d] > 1) o.streaming = 0;
        }
        if (ins[k].data == out->data) o.streaming = 0;  // in-place: keep coherent loads
    }
    for (int i = 0; i < n_instr; i++) p.prog[i] = prog[i];

    // Vector-path eligibility.
    const int last = f.rank - 1;
    const int64_t inner = f.dims[last];
    auto aligned = [&](const void* ptr, int dt, const int64_t* st) {
        int64_t a = 8 * dtype_size(dt);
        if (a > 16) a = 16;
        if ((uintptr_t)ptr % (uintptr_t)a) return false;
        for (int d = 0; d < last; d++)
            if ((st[d] * dtype_size(dt)) % a) return false;
        return true;
    };
    bool vec = f.strides[0][last] == 1 && aligned(out->data, out->dtype, f.strides[0]);
    for (int k = 0; k < n_ins && vec; k++) {
        int64_t s = f.strides[1 + k][last];
        if (s == 1) vec = aligned(ins[k].data, ins[k].dtype, f.strides[1 + k]);
        else if (s == 0) p.in[k].inner_bcast = 1;
        else vec = false;
    }
    if (f.rank > 1 && inner % V) vec = false;
    if (n < V) vec = false;
    // Both paths decompose ELEMENT indices; a vector (V elements, inner % V
    // == 0 when rank > 1) never straddles a row.
    for (int d = 1; d < f.rank; d++) p.dm[d] = DivMod((uint64_t)f.dims[d]);
    p.idx32 = (uint64_t)n < 0xffffffffull ? 1 : 0;
    if (p.idx32) {
        // Largest offset of the output and of each input, with non-negative
        // strides only: below 2^31 everywhere allows 32-bit offset sums.
        bool small = true;
        for (int k = 0; k <= n_ins && small; k++) {
            int64_t top = 0;
            for (int d = 0; d < f.rank && small; d++) {
                const int64_t st = f.strides[k][d];
                if (st < 0 || st > 0x7fffffff) small = false;
                else top += (f.dims[d] - 1) * st;
                if (top > 0x7fffffff) small = false;
            }
        }
        if (small) p.idx32 = 2;
    }

    // Fast math (SFU exp / reciprocal) when an fp32 chain ends in a 16-bit
    // store and every intermediate rounding is to fp32 or coarser: the
    // approximation error is far below the output's half-ulp.
    bool fast = cm == TADMA_COMPUTE_F32 && (out->dtype == TADMA_F16 || out->dtype == TADMA_BF16);
    for (int i = 0; i < n_instr && fast; i++) {
        int rd = prog[i].round_dtype;
        if (!(rd < 0 || rd == TADMA_F32 || rd == TADMA_F16 || rd == TADMA_BF16)) fast = false;
    }
    cudaStream_t s = (cudaStream_t)stream;
    // Narrow operands (fp32 compute): the raw-word kernel keeps more loads in flight.
    bool narrow = vec && cm == TADMA_COMPUTE_F32;
    for (int k = 0; k < n_ins && narrow; k++) {
        const int es = dtype_size(ins[k].dtype);
        narrow = p.in[k].inner_bcast ? (es <= 4 && ins[k].dtype != TADMA_F64 && ins[k].dtype != TADMA_I64) : es <= 2;
    }
    auto go = [&](const ChainParams& pp, bool v, int64_t work) {
        switch (cm) {
        case TADMA_COMPUTE_F32: return launch_interp<float>(n_ins, fast, pp, v, work, s, narrow);
        case TADMA_COMPUTE_F64: return launch_interp<double>(n_ins, false, pp, v, work, s, false);
        default: return launch_interp<int64_t>(n_ins, false, pp, v, work, s, false);
        }
    };
    if (!vec) {
        // A single input whose contiguous dim differs from the output's: tiled transpose.
        int dt_in = -1;
        if (n_ins == 1 && cm == TADMA_COMPUTE_F32 && f.rank >= 2 && f.strides[0][last] == 1 &&
            f.strides[1][last] != 1 && f.strides[1][last] != 0 && ins[0].data != out->data) {
            for (int d = 0; d < last; d++)
                if (f.strides[1][d] == 1) dt_in = d;
        }
        if (dt_in >= 0 && (f.dims[dt_in] + 31) / 32 <= 65535 && (f.dims[last] + 31) / 32 <= 0x7fffffff) {
            TransposeParams tp{};
            tp.in = (const char*)ins[0].data;
            tp.out = (char*)out->data;
            tp.in_dtype = ins[0].dtype;
            tp.out_dtype = out->dtype;
            tp.n_i = f.dims[dt_in];
            tp.n_j = f.dims[last];
            tp.in_sj = f.strides[1][last];
            tp.out_si = f.strides[0][dt_in];
            tp.nbatch = 1;
            for (int d = 0; d < last; d++) {
                if (d == dt_in) continue;
                tp.bdm[tp.nb] = DivMod((uint64_t)f.dims[d]);
                tp.b_in[tp.nb] = f.strides[1][d];
                tp.b_out[tp.nb] = f.strides[0][d];
                tp.nbatch *= f.dims[d];
                tp.nb++;
            }
            tp.chain = p;
            return launch_transpose(fast, tp, s);
        }
        p.start = 0;
        p.n = n;
        return go(p, false, n);
    }
    // Vector path: vector vi covers elements [vi * V, vi * V + V); a rank-1
    // tail of n % V elements goes to the scalar kernel afterwards.
    const int64_t nvec = n / V;
    ChainParams pv = p;
    pv.n = nvec;
    int rc;
    AffineMatch am = cm == TADMA_COMPUTE_F32 ? match_affine(prog, n_instr, n_ins) : AffineMatch{};
    const bool fdt = out->dtype == TADMA_F32 || out->dtype == TADMA_F16 || out->dtype == TADMA_BF16;
    const bool rows_ok = am.ok && am.add && f.rank == 2 && fdt && ins[0].dtype == ins[1].dtype &&
                         (ins[0].dtype == TADMA_F32 || ins[0].dtype == TADMA_F16 || ins[0].dtype == TADMA_BF16) &&
                         (out->dtype == ins[0].dtype || out->dtype == TADMA_F32) && f.strides[2][0] == 0 &&
                         f.strides[2][1] == 1 && f.strides[1][1] == 1 && f.strides[0][1] == 1 && !p.in[1].inner_bcast;
    auto fdt3 = [](int dt) { return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16; };
    bool typed_ok = cm == TADMA_COMPUTE_F32 && (n_ins == 1 || n_ins == 2) && fdt3(out->dtype);
    for (int k = 0; k < n_ins && typed_ok; k++)
        typed_ok = ins[k].dtype == ins[0].dtype && fdt3(ins[k].dtype) && !p.in[k].inner_bcast;
    // One instruction (or none: a cast) whose rounding is a no-op before the store.
    int op1 = -1;
    bool imm1 = false;
    if (typed_ok && n_instr <= 1) {
        const tadma_instr* I = n_instr == 1 ? &prog[0] : nullptr;
        const int rd = I ? I->round_dtype : -1;
        const bool round_ok = rd < 0 || rd == TADMA_F32 || rd == out->dtype;
        if (!I) {
            if (n_ins == 1) op1 = TADMA_OP_COPY;
        } else if (round_ok && I->op == TADMA_OP_COPY && I->b != TADMA_SRC_IMM && n_ins == 1) {
            op1 = TADMA_OP_COPY;
        } else if (round_ok && ins[0].dtype == out->dtype && I->c == TADMA_SRC_NONE &&
                   (I->op == TADMA_OP_ADD || I->op == TADMA_OP_SUB || I->op == TADMA_OP_MUL || I->op == TADMA_OP_DIV ||
                    I->op == TADMA_OP_RSUB || I->op == TADMA_OP_RDIV || I->op == TADMA_OP_MAX || I->op == TADMA_OP_MIN)) {
            if (I->b == TADMA_SRC_IMM && n_ins == 1) {
                op1 = I->op;
                imm1 = true;
            } else if (I->b == 1 && n_ins == 2) {
                op1 = I->op;
            }
        }
    }
    // Comparisons into bool and where(bool / u8, T, T) -> T, one instruction.
    int cmp_op = -1;
    bool cmp_imm = false, where_ok = false;
    if (n_instr == 1 && cm == TADMA_COMPUTE_F32) {
        const tadma_instr& I = prog[0];
        const int rd = I.round_dtype;
        bool no_bcast = true;
        for (int k = 0; k < n_ins; k++) no_bcast = no_bcast && !p.in[k].inner_bcast;
        if (no_bcast && out->dtype == TADMA_BOOL && (rd < 0 || rd == TADMA_BOOL || rd == TADMA_F32) &&
            I.op >= TADMA_OP_EQ && I.op <= TADMA_OP_GE && I.c == TADMA_SRC_NONE && fdt3(ins[0].dtype)) {
            if (I.b == TADMA_SRC_IMM && n_ins == 1) {
                cmp_op = I.op;
                cmp_imm = true;
            } else if (I.b == 1 && n_ins == 2 && ins[1].dtype == ins[0].dtype) {
                cmp_op = I.op;
            }
        }
        where_ok = no_bcast && I.op == TADMA_OP_WHERE && I.b == 1 && I.c == 2 && n_ins == 3 &&
                   (ins[0].dtype == TADMA_BOOL || ins[0].dtype == TADMA_U8) && fdt3(out->dtype) &&
                   ins[1].dtype == out->dtype && ins[2].dtype == out->dtype &&
                   (rd < 0 || rd == TADMA_F32 || rd == out->dtype);
    }
    // First match wins: the row-broadcast affine kernel, the typed single-op
    // kernels, compile-time affine programs, then the interpreted kernels.
    if (rows_ok) {
        // vec eligibility (checked above) already guarantees 16-byte alignment of
        // every row start and inner % 8 == 0.
        AffineRowsParams ap{};
        ap.x = (const char*)ins[0].data;
        ap.bias = (const char*)ins[1].data;
        ap.out = (char*)out->data;
        ap.rows = f.dims[0];
        ap.ncv = f.dims[1] / V;
        ap.x_rs = f.strides[1][0];
        ap.out_rs = f.strides[0][0];
        ap.scale = am.mul ? am.scale : 1.0f;
        rc = launch_rows(ins[0].dtype, out->dtype, am.act, ap, s);
    } else if (cmp_op >= 0) {
        rc = launch_cmp(ins[0].dtype, cmp_op, cmp_imm, pv, nvec, s);
    } else if (where_ok) {
        rc = launch_where(out->dtype, pv, nvec, s);
    } else if (op1 >= 0) {
        rc = launch_typed1(ins[0].dtype, out->dtype, op1, imm1, pv, nvec, s);
    } else if (am.ok) {
        pv.scale = am.scale;
        rc = launch_affine(am.act, fast, am.mul, am.add, pv, nvec, s, narrow);
    } else if (typed_ok) {
        rc = launch_typed(ins[0].dtype, out->dtype, n_ins, fast, pv, nvec, s);
    } else {
        rc = go(pv, true, nvec);
    }
    if (rc != TADMA_OK) return rc;
    if (nvec * V < n) {
        p.start = nvec * V;
        p.n = n;
        return go(p, false, n - nvec * V);
    }
    return TADMA_OK;
}

extern "C" int tadma_b200_reduce_chain(int32_t op, const tadma_tensor* ins, int32_t n_ins, const tadma_instr* prog,
                                       int32_t n_instr, int32_t compute, int32_t axis, const tadma_tensor* out,
                                       void* stream) {
    std::string err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (n_ins < 1 || n_ins > TADMA_MAX_INPUTS) return fail(TADMA_ERR_INVALID, "n_ins out of range [1, 4]");
    if (n_instr < 0 || n_instr > TADMA_MAX_INSTR) return fail(TADMA_ERR_INVALID, "n_instr out of range [0, 16]");
    if (!ins) return fail(TADMA_ERR_INVALID, "ins is NULL");
    if (n_instr > 0 && !prog) return fail(TADMA_ERR_INVALID, "prog is NULL");
    if (op < TADMA_REDUCE_SUM || op > TADMA_REDUCE_RMS) return fail(TADMA_ERR_INVALID, "unknown reduce op");
    const int rank = ins[0].rank;
    if (rank < 1) return fail(TADMA_ERR_INVALID, "ins must have rank >= 1");
    int64_t S[TADMA_MAX_RANK];
    for (int d = 0; d < rank; d++) S[d] = 1;
    for (int k = 0; k < n_ins; k++) {
        err = check_tensor(&ins[k], "ins[k]");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (ins[k].rank != rank) return fail(TADMA_ERR_INVALID, "ins must share one rank");
        for (int d = 0; d < rank; d++) {
            if (ins[k].dims[d] == 1) continue;
            if (S[d] != 1 && S[d] != ins[k].dims[d]) return fail(TADMA_ERR_INVALID, "ins dims do not broadcast");
            S[d] = ins[k].dims[d];
        }
    }
    for (int i = 0; i < n_instr; i++) {
        const tadma_instr& I = prog[i];
        if (!valid_op(I.op)) return fail(TADMA_ERR_INVALID, "unknown op code");
        bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
        if (needs_b && !(I.b == TADMA_SRC_IMM || (I.b >= 0 && I.b < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector b out of range");
        if (I.op == TADMA_OP_WHERE && !(I.c == TADMA_SRC_IMM || (I.c >= 0 && I.c < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector c out of range");
        if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return fail(TADMA_ERR_INVALID, "bad round_dtype");
    }
    const int ax = axis < 0 ? axis + rank : axis;
    if (ax < 0 || ax >= rank) return fail(TADMA_ERR_INVALID, "axis out of range");
    const bool keep = out->rank == rank;
    if (!keep && out->rank != rank - 1) return fail(TADMA_ERR_INVALID, "out rank must be rank or rank - 1");
    for (int d = 0, k = 0; d < rank; d++) {
        if (d == ax) {
            if (keep && out->dims[k++] != 1) return fail(TADMA_ERR_INVALID, "out dims[axis] must be 1");
            continue;
        }
        if (out->dims[k++] != S[d]) return fail(TADMA_ERR_INVALID, "out dims do not match the reduced dims");
    }
    const bool arg = op == TADMA_REDUCE_ARGMAX || op == TADMA_REDUCE_ARGMIN;
    if (arg && out->dtype != TADMA_I64 && out->dtype != TADMA_I32)
        return fail(TADMA_ERR_INVALID, "argmax/argmin output must be int64 or int32");
    // The chain's natural result type decides the compute type, as for a
    // materialised chain (ins[0]'s dtype standing in for the temporary's).
    tadma_tensor chain_out = ins[0];
    int cm = resolve_compute(&chain_out, ins, n_ins, prog, n_instr, compute);
    if (cm < TADMA_COMPUTE_F32 || cm > TADMA_COMPUTE_I64) return fail(TADMA_ERR_INVALID, "bad compute mode");
    if (cm == TADMA_COMPUTE_I64)
        for (int i = 0; i < n_instr; i++)
            if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW)
                return fail(TADMA_ERR_UNSUPPORTED, "transcendental op in int64 compute");
    const int64_t R = S[ax];
    if (R == 0 && op != TADMA_REDUCE_SUM && op != TADMA_REDUCE_SUMSQ)
        return fail(TADMA_ERR_INVALID, "empty reduction has no identity for this op");
    if (numel(out) == 0) return TADMA_OK;

    ChainReduceParams p{};
    p.chain.n_instr = n_instr;
    for (int i = 0; i < n_instr; i++) p.chain.prog[i] = prog[i];
    p.n_ins = n_ins;
    p.R = R;
    p.out = (char*)out->data;
    p.out_dtype = out->dtype;
    p.square = (op == TADMA_REDUCE_SUMSQ || op == TADMA_REDUCE_RMS) ? 1 : 0;
    p.post = op == TADMA_REDUCE_MEAN ? POST_MEAN : op == TADMA_REDUCE_RMS ? POST_RMS : POST_NONE;
    const int kind = op == TADMA_REDUCE_MAX ? K_MAX : op == TADMA_REDUCE_MIN ? K_MIN
                   : op == TADMA_REDUCE_ARGMAX ? K_ARGMAX : op == TADMA_REDUCE_ARGMIN ? K_ARGMIN : K_SUM;
    // Kept dims, folded jointly for the operands and out.
    int64_t kd[TADMA_MAX_RANK], ks[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    int kr = 0;
    for (int d = 0; d < rank; d++) {
        if (d == ax) continue;
        kd[kr] = S[d];
        ks[0][kr] = out->strides[keep ? d : (d < ax ? d : d - 1)];
        for (int k = 0; k < n_ins; k++) ks[1 + k][kr] = ins[k].dims[d] == 1 ? 0 : ins[k].strides[d];
        kr++;
    }
    int64_t nrows = 1;
    Folded f{};
    if (kr > 0) {
        f = fold(kr, kd, ks, 1 + n_ins);
        for (int d = 0; d < f.rank; d++) nrows *= f.dims[d];
    }
    p.nrows = nrows;
    p.krank = kr > 0 ? f.rank : 0;
    for (int d = 0; d < p.krank; d++) {
        p.kdm[d] = DivMod((uint64_t)f.dims[d]);
        p.kout[d] = f.strides[0][d];
        for (int k = 0; k < n_ins; k++) p.kin[k][d] = f.strides[1 + k][d];
    }
    bool vec = cm == TADMA_COMPUTE_F32 && R >= V;
    for (int k = 0; k < n_ins; k++) {
        Operand& o = p.chain.in[k];
        o.base = (const char*)ins[k].data;
        o.dtype = ins[k].dtype;
        o.streaming = 0;
        p.ax[k] = ins[k].dims[ax] == 1 ? 0 : ins[k].strides[ax];
        o.inner_bcast = p.ax[k] == 0 ? 1 : 0;
        if (p.ax[k] == 0) continue;
        const int es = dtype_size(o.dtype);
        const bool vdt = o.dtype == TADMA_F32 || o.dtype == TADMA_F16 || o.dtype == TADMA_BF16;
        bool ok = vdt && p.ax[k] == 1 && (uintptr_t)o.base % 16 == 0;
        for (int d = 0; d < p.krank && ok; d++) ok = (p.kin[k][d] * es) % 16 == 0;
        vec = vec && ok;
    }
    cudaStream_t s = (cudaStream_t)stream;
    switch (cm) {
    case TADMA_COMPUTE_F32:
        return vec ? launch_chain_reduce<float, true>(kind, p, s) : launch_chain_reduce<float, false>(kind, p, s);
    case TADMA_COMPUTE_F64: return launch_chain_reduce<double, false>(kind, p, s);
    default: return launch_chain_reduce<int64_t, false>(kind, p, s);
    }
}
