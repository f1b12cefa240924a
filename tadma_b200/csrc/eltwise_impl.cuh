// eltwise_impl.cuh - fused element-wise / broadcast engine (sm_100a): the
// types, device helpers and chain kernels shared by its translation units
// (eltwise.cu: entry points and dispatch; eltwise_interp_*.cu, eltwise_affine.cu,
// eltwise_typed.cu, eltwise_transpose.cu, chain_reduce.cu: kernel families).
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
#pragma once

#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"
#include "fprog.cuh"
#include "layout.hpp"
#include "ops.cuh"
#include "reduce_state.cuh"

namespace tadma_b200 {

constexpr int V = 8;        // elements per vector step
// Vector steps in flight per thread: 2, or 1 with 3-6 operands (their
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
    int32_t pad2;
    FProg fp;     // the program pre-decoded for the typed fp32 kernels
};

// Program selector of a kernel instance: the run-time interpreter (precise or
// fast math) or a compile-time affine + activation chain act(x * s + b).
constexpr int PROG_INTERP = 0;
constexpr int PROG_INTERP_FAST = 1;
constexpr int ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2, ACT_SIGMOID = 3, ACT_TANH = 4;
constexpr int affine_prog(int act, bool fast, bool mul, bool add) {
    return 0x100 | (act << 4) | (fast ? 4 : 0) | (mul ? 2 : 0) | (add ? 1 : 0);
}

struct AffineRowsParams {
    const char* x;
    const char* bias;
    char* out;
    int64_t rows, ncv;      // rows, 8-element column vectors
    int64_t x_rs, out_rs;   // row strides (elements)
    float scale;
};

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
    PostChain pc;  // applied to each reduced value before its store (n = 0: none)
};

constexpr int POST_NONE = 0, POST_MEAN = 1, POST_RMS = 2;

// Launchers of the kernel families, one translation unit each.
int blocks_per_sm(const void* fn);
// Interpreter launch; `fast` and `narrow` only exist for fp32 compute.
int launch_interp_f32(int nin, bool fast, const ChainParams& p, bool vec, int64_t work, cudaStream_t s, bool narrow);
int launch_interp_f64(int nin, const ChainParams& p, bool vec, int64_t work, cudaStream_t s);
int launch_interp_i64(int nin, const ChainParams& p, bool vec, int64_t work, cudaStream_t s);
int launch_affine(int act, bool fast, bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s,
                  bool narrow);
int launch_typed1(int idt, int odt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s);
int launch_cmp(int idt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s);
int launch_where(int dt, const ChainParams& p, int64_t nvec, cudaStream_t s);
// One-dtype chains (fp32 compute, every operand of dtype idt, F32 / F16 /
// BF16) on the pre-decoded program p.fp: p.in[0 .. nv) contiguous along the
// innermost folded dim, p.in[nv .. nv + ns) broadcast along it; 1 <= nv,
// ns <= 2, nv + ns <= 6 (else TADMA_ERR_UNSUPPORTED, nothing launched).
int launch_typed(int idt, int odt, int nv, int ns, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s);
int launch_rows(int xdt, int odt, int act, const AffineRowsParams& p, cudaStream_t s);
int launch_transpose(bool fast, const TransposeParams& tp, cudaStream_t s);
int launch_chain_reduce_f32(int kind, bool vec, const ChainReduceParams& p, cudaStream_t s);
// fp32 compute, every operand streamed along the axis with dtype dt (F32 / F16
// / BF16) or broadcast along it; runs the pre-decoded program p.chain.fp.
int launch_chain_reduce_typed(int kind, int dt, const ChainReduceParams& p, cudaStream_t s);
int launch_chain_reduce_f64(int kind, const ChainReduceParams& p, cudaStream_t s);
int launch_chain_reduce_i64(int kind, const ChainReduceParams& p, cudaStream_t s);
// reduce.cu: a chain reduction of the form sq(pre(op1(x, m))) with m one value
// per output row, on the reduction engine's row kernel (TADMA_ERR_UNSUPPORTED
// when the layout is not its own; nothing recorded then).
int reduce_rowop(int32_t op, const int64_t* shape, int32_t rank, int32_t ax, const tadma_tensor* in, int32_t op1,
                 const tadma_tensor* rop, double imm1, int32_t pre_op, int32_t square, const tadma_instr* post,
                 int32_t n_post, const tadma_tensor* out, cudaStream_t s);

namespace {

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

// Raw bits of a double / int64 value rounded once to fp16 or bf16.
__device__ __forceinline__ uint32_t h16_bits(double v, int dt) {
    return dt == TADMA_F16 ? (uint32_t)__half_as_ushort(d2h(v)) : (uint32_t)__bfloat16_as_ushort(d2bf(v));
}
__device__ __forceinline__ uint32_t h16_bits(int64_t v, int dt) {
    return dt == TADMA_F16 ? (uint32_t)__half_as_ushort(__ll2half_rn(v)) : (uint32_t)__bfloat16_as_ushort(__ll2bfloat16_rn(v));
}

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
            if constexpr (std::is_same<C, float>::value) {
                st_stream_v4(p, pack8(v, dt));
            } else {
                // double / int64 values round once to the 16-bit type
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < V; j += 2) {
                    const uint32_t lo = h16_bits(v[j], dt), hi = h16_bits(v[j + 1], dt);
                    w[j / 2] = lo | (hi << 16);
                }
                st_stream_v4(p, make_uint4(w[0], w[1], w[2], w[3]));
            }
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

}  // namespace
}  // namespace tadma_b200
