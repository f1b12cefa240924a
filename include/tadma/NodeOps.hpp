// NodeOps.hpp - operators on tensors handed out by an ExecutionTape.
//
// In the reference every operator builds a node (Tensor.hpp:494-540,
// Operations.hpp:166-188).  In this library the operators on ordinary tensors
// compute at once (Operations.hpp); on a tape tensor (TapeTensor: its inputs
// are only produced when the tape runs) the same spellings build the
// reference's nodes instead, with device-capable functors, so a chain of them
// appended to a tape merges into one kernel.  These overloads are more
// constrained than the eager ones and win whenever an operand is a tape
// tensor.  Element math runs in fp32 for 16-bit values, in the value's type
// otherwise; result types follow the functor (Kernels.hpp:20-45).
#pragma once

#include <cmath>

#include "ExecutionTape.hpp"
#include "Operations.hpp"

namespace tadma {
namespace nodefn {

template <typename T>
__host__ __device__ inline auto up(const T& x) {
    if constexpr (std::is_same_v<T, __half> || std::is_same_v<T, __nv_bfloat16>) return (float)x;
    else return x;
}

#define TADMA_NODE_SCALAR(Name, expr)                                               \
    template <typename S>                                                           \
    struct Name {                                                                   \
        S v;                                                                        \
        static constexpr bool tadma_device = true;                                  \
        template <typename X>                                                       \
        __host__ __device__ auto operator()(const X& x_) const {                    \
            const auto x = up(x_);                                                  \
            return expr;                                                            \
        }                                                                           \
    };
TADMA_NODE_SCALAR(AddS, x + v)
TADMA_NODE_SCALAR(SubS, x - v)
TADMA_NODE_SCALAR(MulS, x * v)
TADMA_NODE_SCALAR(DivS, x / v)
TADMA_NODE_SCALAR(RSubS, v - x)
TADMA_NODE_SCALAR(RDivS, v / x)
TADMA_NODE_SCALAR(GtS, x > v)
TADMA_NODE_SCALAR(LtS, x < v)
TADMA_NODE_SCALAR(EqS, x == v)
TADMA_NODE_SCALAR(NeS, x != v)
TADMA_NODE_SCALAR(PowS, pow_(x, v))
#undef TADMA_NODE_SCALAR

#define TADMA_NODE_BINARY(Name, Comm, expr)                                         \
    struct Name {                                                                   \
        static constexpr bool tadma_device = true;                                  \
        static constexpr bool commutative = Comm;                                   \
        template <typename A, typename B>                                           \
        __host__ __device__ auto operator()(const A& a_, const B& b_) const {       \
            const auto a = up(a_);                                                  \
            const auto b = up(b_);                                                  \
            return expr;                                                            \
        }                                                                           \
    };
TADMA_NODE_BINARY(Add, true, a + b)
TADMA_NODE_BINARY(Sub, false, a - b)
TADMA_NODE_BINARY(Mul, true, a * b)
TADMA_NODE_BINARY(Div, false, a / b)
TADMA_NODE_BINARY(Gt, false, a > b)
TADMA_NODE_BINARY(Lt, false, a < b)
TADMA_NODE_BINARY(Eq, true, a == b)
TADMA_NODE_BINARY(Ne, true, a != b)
TADMA_NODE_BINARY(And, true, a & b)
TADMA_NODE_BINARY(Or, true, a | b)
TADMA_NODE_BINARY(Xor, true, a ^ b)
TADMA_NODE_BINARY(LAnd, true, a && b)
TADMA_NODE_BINARY(LOr, true, a || b)
#undef TADMA_NODE_BINARY

// Math on fp32 (16-bit and fp32 values) or fp64 (double and integers), as
// std::name would pick it.
#define TADMA_NODE_MATH(name)                                                       \
    template <typename X>                                                           \
    __host__ __device__ inline auto name##_(const X& x) {                          \
        if constexpr (std::is_same_v<X, float>) return ::name##f(x);               \
        else return ::name((double)x);                                              \
    }
TADMA_NODE_MATH(sin)
TADMA_NODE_MATH(cos)
TADMA_NODE_MATH(tan)
TADMA_NODE_MATH(asin)
TADMA_NODE_MATH(acos)
TADMA_NODE_MATH(atan)
TADMA_NODE_MATH(asinh)
TADMA_NODE_MATH(acosh)
TADMA_NODE_MATH(atanh)
TADMA_NODE_MATH(exp)
TADMA_NODE_MATH(log)
TADMA_NODE_MATH(sqrt)
TADMA_NODE_MATH(erf)
TADMA_NODE_MATH(tanh)
#undef TADMA_NODE_MATH

template <typename X, typename S>
__host__ __device__ inline auto pow_(const X& x, const S& s) {
    if constexpr (std::is_same_v<X, float> && !std::is_same_v<S, double>) return ::powf(x, (float)s);
    else return ::pow((double)x, (double)s);
}

#define TADMA_NODE_UNARY(Name, expr)                                                \
    struct Name {                                                                   \
        static constexpr bool tadma_device = true;                                  \
        template <typename X_>                                                      \
        __host__ __device__ auto operator()(const X_& x_) const {                   \
            const auto x = up(x_);                                                  \
            using X = std::decay_t<decltype(x)>;                                    \
            (void)sizeof(X);                                                        \
            return expr;                                                            \
        }                                                                           \
    };
TADMA_NODE_UNARY(Neg, -x)
TADMA_NODE_UNARY(Abs, x < X(0) ? -x : x)
TADMA_NODE_UNARY(Sin, sin_(x))
TADMA_NODE_UNARY(Cos, cos_(x))
TADMA_NODE_UNARY(Tan, tan_(x))
TADMA_NODE_UNARY(Asin, asin_(x))
TADMA_NODE_UNARY(Acos, acos_(x))
TADMA_NODE_UNARY(Atan, atan_(x))
TADMA_NODE_UNARY(Asinh, asinh_(x))
TADMA_NODE_UNARY(Acosh, acosh_(x))
TADMA_NODE_UNARY(Atanh, atanh_(x))
TADMA_NODE_UNARY(Exp, exp_(x))
TADMA_NODE_UNARY(Log, log_(x))
TADMA_NODE_UNARY(Sqrt, sqrt_(x))
TADMA_NODE_UNARY(Erf, erf_(x))
TADMA_NODE_UNARY(Relu, x > X(0) ? x : X(0))
TADMA_NODE_UNARY(Sigmoid, 1 / (1 + exp_(-x)))
TADMA_NODE_UNARY(Tanh, tanh_(x))
// 0.5 x (1 + tanh(u)) of Operations.hpp:181, in double as there (0.5 is a
// double literal), written x / (1 + e^(-2u)): the same function without the
// cancellation below x = -3.
TADMA_NODE_UNARY(Gelu, (double)x / (1.0 + ::exp(-2.0 * (0.7978845608 * ((double)x + 0.044715 * (double)x * (double)x * (double)x)))))
TADMA_NODE_UNARY(Negate, -x)
#undef TADMA_NODE_UNARY

}  // namespace nodefn

// tensor (op) scalar, scalar (op) tensor
template <TapeTensor T, Scalar S> auto operator+(const T& t, S v) { return EltwiseNode(t, nodefn::AddS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator-(const T& t, S v) { return EltwiseNode(t, nodefn::SubS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator*(const T& t, S v) { return EltwiseNode(t, nodefn::MulS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator/(const T& t, S v) { return EltwiseNode(t, nodefn::DivS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator-(S v, const T& t) { return EltwiseNode(t, nodefn::RSubS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator/(S v, const T& t) { return EltwiseNode(t, nodefn::RDivS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator+(S v, const T& t) { return EltwiseNode(t, nodefn::AddS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator*(S v, const T& t) { return EltwiseNode(t, nodefn::MulS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator>(const T& t, S v) { return EltwiseNode(t, nodefn::GtS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator<(const T& t, S v) { return EltwiseNode(t, nodefn::LtS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator==(const T& t, S v) { return EltwiseNode(t, nodefn::EqS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator!=(const T& t, S v) { return EltwiseNode(t, nodefn::NeS<scalar_t<S>>{(scalar_t<S>)v}); }

// tensor (op) tensor, when either side is a tape tensor
#define TADMA_TAPE_BINARY(op, Fn)                                                   \
    template <AnyTensor A, AnyTensor B>                                             \
        requires(TapeTensor<A> || TapeTensor<B>)                                    \
    auto operator op(const A& a, const B& b) {                                      \
        return CombineToNode(a, b, nodefn::Fn{});                                   \
    }
TADMA_TAPE_BINARY(+, Add)
TADMA_TAPE_BINARY(-, Sub)
TADMA_TAPE_BINARY(*, Mul)
TADMA_TAPE_BINARY(/, Div)
TADMA_TAPE_BINARY(>, Gt)
TADMA_TAPE_BINARY(<, Lt)
TADMA_TAPE_BINARY(==, Eq)
TADMA_TAPE_BINARY(!=, Ne)
TADMA_TAPE_BINARY(&, And)
TADMA_TAPE_BINARY(|, Or)
TADMA_TAPE_BINARY(^, Xor)
TADMA_TAPE_BINARY(&&, LAnd)
TADMA_TAPE_BINARY(||, LOr)
#undef TADMA_TAPE_BINARY

template <TapeTensor T> auto operator-(const T& t) { return EltwiseNode(t, nodefn::Neg{}); }

// compound assignment: x = f(x, y) in place (CombineNode / InplaceNode)
template <TapeTensor T, Scalar S> auto operator+=(T& t, S v) { return InplaceNode(t, nodefn::AddS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator-=(T& t, S v) { return InplaceNode(t, nodefn::SubS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator*=(T& t, S v) { return InplaceNode(t, nodefn::MulS<scalar_t<S>>{(scalar_t<S>)v}); }
template <TapeTensor T, Scalar S> auto operator/=(T& t, S v) { return InplaceNode(t, nodefn::DivS<scalar_t<S>>{(scalar_t<S>)v}); }
#define TADMA_TAPE_COMPOUND(op, Fn)                                                 \
    template <AnyTensor A, AnyTensor B>                                             \
        requires(TapeTensor<A> || TapeTensor<B>)                                    \
    auto operator op(A& a, const B& b) {                                            \
        return CombineNode(a, b, nodefn::Fn{});                                     \
    }
TADMA_TAPE_COMPOUND(+=, Add)
TADMA_TAPE_COMPOUND(-=, Sub)
TADMA_TAPE_COMPOUND(*=, Mul)
TADMA_TAPE_COMPOUND(/=, Div)
TADMA_TAPE_COMPOUND(&=, And)
TADMA_TAPE_COMPOUND(|=, Or)
TADMA_TAPE_COMPOUND(^=, Xor)
#undef TADMA_TAPE_COMPOUND

// MKOP unary ops (Operations.hpp:166-182); Inplace = true rewrites t.
#define TADMA_TAPE_MKOP(name, Fn)                                                   \
    template <bool Inplace = true, TapeTensor T>                                    \
    auto name(T&& t) {                                                              \
        return MakeEltwiseNode<Inplace>(t, nodefn::Fn{});                           \
    }
TADMA_TAPE_MKOP(abs, Abs)
TADMA_TAPE_MKOP(sin, Sin)
TADMA_TAPE_MKOP(cos, Cos)
TADMA_TAPE_MKOP(tan, Tan)
TADMA_TAPE_MKOP(asin, Asin)
TADMA_TAPE_MKOP(acos, Acos)
TADMA_TAPE_MKOP(atan, Atan)
TADMA_TAPE_MKOP(asinh, Asinh)
TADMA_TAPE_MKOP(acosh, Acosh)
TADMA_TAPE_MKOP(atanh, Atanh)
TADMA_TAPE_MKOP(exp, Exp)
TADMA_TAPE_MKOP(log, Log)
TADMA_TAPE_MKOP(sqrt, Sqrt)
TADMA_TAPE_MKOP(erf, Erf)
TADMA_TAPE_MKOP(relu, Relu)
TADMA_TAPE_MKOP(sigmoid, Sigmoid)
TADMA_TAPE_MKOP(tanh, Tanh)
TADMA_TAPE_MKOP(gelu, Gelu)
TADMA_TAPE_MKOP(negate, Negate)
#undef TADMA_TAPE_MKOP

template <bool Inplace = true, TapeTensor T, Scalar S>
auto pow(T&& t, S s) {
    return MakeEltwiseNode<Inplace>(t, nodefn::PowS<scalar_t<S>>{(scalar_t<S>)s});
}

}  // namespace tadma
