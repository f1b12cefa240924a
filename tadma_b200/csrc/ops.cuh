// ops.cuh - scalar bodies of the element-wise op codes (tadma_op), shared
// by the chain engine and the reduction pre-op.  fp32 arithmetic uses the
// explicit round-to-nearest intrinsics so no multiply-add is contracted: each
// op rounds once, as each reference node writes a rounded tensor.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace tadma_b200 {
namespace {

__device__ __forceinline__ float gelu_f(float x) {
    // 0.5 x (1 + tanh(u)) == x * sigmoid(2u) == x / (1 + exp(-2u)), with
    // u = 0.7978845608 (x + 0.044715 x^3) (Operations.hpp:181).  This form has
    // no inf/inf for large |u|, unlike the reference's tanh (Operations.hpp:160-164).
    float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    float u = __fmul_rn(0.7978845608f, __fadd_rn(x, x3));
    float e = expf(__fmul_rn(-2.0f, u));
    return __fdiv_rn(x, __fadd_rn(1.0f, e));
}

// Fast forms, used when an fp32 chain writes a 16-bit output: the SFU
// base-2 exponential and reciprocal (ex2.approx, max relative error ~2^-22;
// rcp.approx, max 1 ulp over the full range), with no branch or select:
//   sigmoid(w / log2 e) = 1 / (1 + 2^(-w)).
// For w << 0 the sum is huge or +inf and the reciprocal goes to 0 as the
// function does; the error stays orders of magnitude below half an
// fp16/bf16 ulp wherever the result is a normal number.
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// sigmoid of w / log2(e): callers fold log2(e) into their own constants.
__device__ __forceinline__ float sigmoid_log2(float w) { return rcp_approx(1.0f + ex2_approx(-w)); }

__device__ __forceinline__ float sigmoid_fast(float y) { return sigmoid_log2(y * 1.4426950408889634f); }

__device__ __forceinline__ float gelu_fast(float x) {
    // gelu(x) = x * sigmoid(2u), u = 0.7978845608 (x + 0.044715 x^3)
    // 2u log2(e) = x (K1 + K3 x^2) with the constants folded.
    constexpr float K1 = 2.0f * 0.7978845608f * 1.4426950408889634f;
    constexpr float K3 = K1 * 0.044715f;
    return x * sigmoid_log2(x * fmaf(K3, x * x, K1));
}

// Rarely fused, register-hungry functions (trig slow paths, erf, log, pow)
// live out of line so they do not inflate the register budget of the chain.
__device__ __noinline__ float unary_cold(int op, float a) {
    switch (op) {
    case TADMA_OP_LOG: return logf(a);
    case TADMA_OP_SIN: return sinf(a);
    case TADMA_OP_COS: return cosf(a);
    case TADMA_OP_TAN: return tanf(a);
    case TADMA_OP_ASIN: return asinf(a);
    case TADMA_OP_ACOS: return acosf(a);
    case TADMA_OP_ATAN: return atanf(a);
    case TADMA_OP_ASINH: return asinhf(a);
    case TADMA_OP_ACOSH: return acoshf(a);
    case TADMA_OP_ATANH: return atanhf(a);
    case TADMA_OP_ERF: return erff(a);
    }
    return a;
}

__device__ __noinline__ float pow_cold(float a, float b) { return powf(a, b); }

template <bool FAST = false>
__device__ __forceinline__ float unary(int op, float a) {
    switch (op) {
    case TADMA_OP_COPY: return a;
    case TADMA_OP_NEG: return -a;
    case TADMA_OP_ABS: return fabsf(a);
    case TADMA_OP_EXP: return FAST ? __expf(a) : expf(a);
    case TADMA_OP_SQRT: return __fsqrt_rn(a);
    case TADMA_OP_RELU: return a > 0.0f ? a : 0.0f;
    case TADMA_OP_SIGMOID: return FAST ? sigmoid_fast(a) : __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-a)));
    case TADMA_OP_TANH: return tanhf(a);
    case TADMA_OP_GELU: return FAST ? gelu_fast(a) : gelu_f(a);
    case TADMA_OP_NOT: return a == 0.0f ? 1.0f : 0.0f;
    }
    return unary_cold(op, a);
}

__device__ __noinline__ double unary_cold(int op, double a) {
    switch (op) {
    case TADMA_OP_LOG: return log(a);
    case TADMA_OP_SIN: return sin(a);
    case TADMA_OP_COS: return cos(a);
    case TADMA_OP_TAN: return tan(a);
    case TADMA_OP_ASIN: return asin(a);
    case TADMA_OP_ACOS: return acos(a);
    case TADMA_OP_ATAN: return atan(a);
    case TADMA_OP_ASINH: return asinh(a);
    case TADMA_OP_ACOSH: return acosh(a);
    case TADMA_OP_ATANH: return atanh(a);
    case TADMA_OP_ERF: return erf(a);
    case TADMA_OP_EXP: return exp(a);
    case TADMA_OP_TANH: return tanh(a);
    }
    return a;
}

__device__ __noinline__ double pow_cold(double a, double b) { return pow(a, b); }

__device__ __noinline__ double gelu_d(double x) {
    // Same stable form as gelu_f: x / (1 + exp(-2u)) == 0.5 x (1 + tanh(u)).
    double u = 0.7978845608 * (x + 0.044715 * x * x * x);
    return x / (1.0 + exp(-2.0 * u));
}

template <bool FAST = false>
__device__ __forceinline__ double unary(int op, double a) {
    switch (op) {
    case TADMA_OP_COPY: return a;
    case TADMA_OP_NEG: return -a;
    case TADMA_OP_ABS: return fabs(a);
    case TADMA_OP_SQRT: return __dsqrt_rn(a);
    case TADMA_OP_RELU: return a > 0.0 ? a : 0.0;
    case TADMA_OP_SIGMOID: return 1.0 / (1.0 + unary_cold(TADMA_OP_EXP, -a));
    case TADMA_OP_GELU: return gelu_d(a);
    case TADMA_OP_NOT: return a == 0.0 ? 1.0 : 0.0;
    }
    return unary_cold(op, a);
}

template <bool FAST = false>
__device__ __forceinline__ int64_t unary(int op, int64_t a) {
    switch (op) {
    case TADMA_OP_NEG: return (int64_t)(0ull - (uint64_t)a);
    case TADMA_OP_ABS: return a < 0 ? (int64_t)(0ull - (uint64_t)a) : a;
    case TADMA_OP_RELU: return a > 0 ? a : 0;
    case TADMA_OP_NOT: return a == 0;
    }
    return a;
}

__device__ __forceinline__ float binary(int op, float a, float b, float c) {
    switch (op) {
    case TADMA_OP_ADD: return __fadd_rn(a, b);
    case TADMA_OP_SUB: return __fsub_rn(a, b);
    case TADMA_OP_MUL: return __fmul_rn(a, b);
    case TADMA_OP_DIV: return __fdiv_rn(a, b);
    case TADMA_OP_POW: return b == 2.0f ? __fmul_rn(a, a) : pow_cold(a, b);
    case TADMA_OP_RSUB: return __fsub_rn(b, a);
    case TADMA_OP_RDIV: return __fdiv_rn(b, a);
    case TADMA_OP_MAX: return (a < b) ? b : a;
    case TADMA_OP_MIN: return (b < a) ? b : a;
    case TADMA_OP_EQ: return a == b;
    case TADMA_OP_NE: return a != b;
    case TADMA_OP_LT: return a < b;
    case TADMA_OP_GT: return a > b;
    case TADMA_OP_LE: return a <= b;
    case TADMA_OP_GE: return a >= b;
    case TADMA_OP_AND: case TADMA_OP_LAND: return (a != 0.0f) && (b != 0.0f);
    case TADMA_OP_OR: case TADMA_OP_LOR: return (a != 0.0f) || (b != 0.0f);
    case TADMA_OP_XOR: return (a != 0.0f) != (b != 0.0f);
    case TADMA_OP_WHERE: return a != 0.0f ? b : c;
    }
    return a;
}

__device__ __forceinline__ double binary(int op, double a, double b, double c) {
    switch (op) {
    case TADMA_OP_ADD: return __dadd_rn(a, b);
    case TADMA_OP_SUB: return __dsub_rn(a, b);
    case TADMA_OP_MUL: return __dmul_rn(a, b);
    case TADMA_OP_DIV: return __ddiv_rn(a, b);
    case TADMA_OP_POW: return b == 2.0 ? __dmul_rn(a, a) : pow_cold(a, b);
    case TADMA_OP_RSUB: return __dsub_rn(b, a);
    case TADMA_OP_RDIV: return __ddiv_rn(b, a);
    case TADMA_OP_MAX: return (a < b) ? b : a;
    case TADMA_OP_MIN: return (b < a) ? b : a;
    case TADMA_OP_EQ: return a == b;
    case TADMA_OP_NE: return a != b;
    case TADMA_OP_LT: return a < b;
    case TADMA_OP_GT: return a > b;
    case TADMA_OP_LE: return a <= b;
    case TADMA_OP_GE: return a >= b;
    case TADMA_OP_AND: case TADMA_OP_LAND: return (a != 0.0) && (b != 0.0);
    case TADMA_OP_OR: case TADMA_OP_LOR: return (a != 0.0) || (b != 0.0);
    case TADMA_OP_XOR: return (a != 0.0) != (b != 0.0);
    case TADMA_OP_WHERE: return a != 0.0 ? b : c;
    }
    return a;
}

__device__ __forceinline__ int64_t binary(int op, int64_t a, int64_t b, int64_t c) {
    switch (op) {
    case TADMA_OP_ADD: return (int64_t)((uint64_t)a + (uint64_t)b);
    case TADMA_OP_SUB: return (int64_t)((uint64_t)a - (uint64_t)b);
    case TADMA_OP_MUL: return (int64_t)((uint64_t)a * (uint64_t)b);
    case TADMA_OP_DIV: return b == 0 ? 0 : (b == -1 ? (int64_t)(0ull - (uint64_t)a) : a / b);
    case TADMA_OP_RSUB: return (int64_t)((uint64_t)b - (uint64_t)a);
    case TADMA_OP_RDIV: return a == 0 ? 0 : (a == -1 ? (int64_t)(0ull - (uint64_t)b) : b / a);
    case TADMA_OP_MAX: return (a < b) ? b : a;
    case TADMA_OP_MIN: return (b < a) ? b : a;
    case TADMA_OP_EQ: return a == b;
    case TADMA_OP_NE: return a != b;
    case TADMA_OP_LT: return a < b;
    case TADMA_OP_GT: return a > b;
    case TADMA_OP_LE: return a <= b;
    case TADMA_OP_GE: return a >= b;
    case TADMA_OP_AND: return a & b;
    case TADMA_OP_OR: return a | b;
    case TADMA_OP_XOR: return a ^ b;
    case TADMA_OP_LAND: return (a != 0) && (b != 0);
    case TADMA_OP_LOR: return (a != 0) || (b != 0);
    case TADMA_OP_WHERE: return a != 0 ? b : c;
    }
    return a;
}

// A reduction's post chain: instructions with immediate operands only,
// applied to each reduced value before its store -- ReduceKernel's post
// functor (kernels/Reduce.hpp:29-56; e.g. the + eps and sqrt that turn a
// variance into layer_norm's denominator, Operations.hpp:195-203) as a chain.
struct PostChain {
    int32_t n;
    int32_t pad;
    tadma_instr prog[TADMA_MAX_INSTR];
};

template <typename C>
__device__ __forceinline__ C post_imm(double v) {
    if constexpr (std::is_same<C, float>::value) return __double2float_rn(v);
    else if constexpr (std::is_same<C, double>::value) return v;
    else return __double2ll_rz(v);
}

template <typename C>
__device__ __forceinline__ C apply_post(const PostChain& pc, C v) {
    for (int i = 0; i < pc.n; i++) {
        const tadma_instr& I = pc.prog[i];
        const C imm = post_imm<C>(I.imm);
        if (I.op < 32) v = I.op == TADMA_OP_COPY ? (I.b == TADMA_SRC_IMM ? imm : v) : unary<false>(I.op, v);
        else v = binary(I.op, v, imm, imm);
        if (I.round_dtype >= 0) v = round_to(v, I.round_dtype);
    }
    return v;
}

}  // namespace
}  // namespace tadma_b200
