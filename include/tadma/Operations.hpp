// Operations.hpp - the Tensor API's operators and free functions, each one
// call into libtadma_b200.so on tadma::stream.
//
// Mirrors include/tadma/Operations.hpp and the operator block of
// include/tadma/Tensor.hpp:494-540 of the reference:
// * tensor (op) scalar, scalar (op) tensor, tensor (op) tensor with the
//   reference's broadcast rule and commutative-operand swap (CombineToNode,
//   Kernels.hpp:33-45), comparisons, bitwise / logical ops, compound
//   assignment in place (InplaceNode / CombineNode, Kernels.hpp:16-31);
// * the MKOP unary set abs ... negate, pow, with `Inplace = true` as the
//   default (Operations.hpp:166-188);
// * softmax, mean_stddev, layer_norm, rms_norm, where, gather, concat
//   (Operations.hpp:190-287) on the fused kernels.
// Result element types follow the C++ the reference evaluates: a bf16 tensor
// times a float scalar is a float tensor, gelu<false> of a float tensor is a
// double tensor (0.5 is a double literal), comparisons give bool.  Each call
// materialises its result, as each reference node does; multi-op fusion is
// available through tadma::fused (a chain of up to 16 ops, one kernel).
#pragma once

#include <utility>

#include "Tensor.hpp"

namespace tadma {

// --------------------------------------------------------- result types --

template <typename T>
constexpr bool is16_v = std::is_same_v<T, __half> || std::is_same_v<T, __nv_bfloat16>;
template <typename T>
constexpr bool isfloat_v = std::is_floating_point_v<T> || is16_v<T>;

namespace detail {
template <typename A, typename B>
auto arith_impl() {
    if constexpr (std::is_same_v<A, double> || std::is_same_v<B, double>) return double{};
    else if constexpr (std::is_same_v<A, float> || std::is_same_v<B, float>) return float{};
    else if constexpr (is16_v<A> && is16_v<B>) {
        if constexpr (std::is_same_v<A, B>) return A{};
        else return float{};
    } else if constexpr (is16_v<A>) return A{};
    else if constexpr (is16_v<B>) return B{};
    else return decltype(A() + B()){};
}
}  // namespace detail

// decltype(a (op) b) as the reference's lambdas compute it.
template <typename A, typename B>
using arith_t = decltype(detail::arith_impl<A, B>());
// std::exp & co. of a 16-bit / float value is float, of double / integer double.
template <typename T>
using math_t = std::conditional_t<std::is_same_v<T, double> || std::is_integral_v<T>, double, float>;

// ------------------------------------------------------------ elementwise --

namespace detail {

template <AnyTensor T>
auto alloc_like_dims(auto value_tag) {
    using V = decltype(value_tag);
    return Tensor<V, Allocator<kCUDA>, typename T::Dims>();
}

// EltwiseNode (Kernels.hpp:20-26): y = f(x) into a new tensor of type R.
template <typename R, AnyTensor T>
auto unary_new(const T& x, int op, double imm = 0.0, int b = TADMA_SRC_NONE) {
    Tensor<R, Allocator<kCUDA>, typename T::Dims> y;
    chain(y, {ins(op, b, imm, dtype_v<R>)}, x);
    return y;
}

// InplaceNode (Kernels.hpp:16-18): x = f(x) over x with its fake dims removed.
template <AnyTensor T>
void unary_inplace(const T& x, int op, double imm = 0.0, int b = TADMA_SRC_NONE) {
    auto v = x.removeFakeDims();
    chain(v, {ins(op, b, imm, dtype_v<typename T::ValueType>)}, v);
}

// CombineToNode (Kernels.hpp:33-45): z = f(x, broadcast(y)) with z of x's dims;
// commutative ops swap the operands when only x broadcasts to y.
template <int OP, bool Commutes, bool Bool, AnyTensor A, AnyTensor B>
auto combine_to(const A& x, const B& y) {
    if constexpr (Commutes && !Broadcastable<B, A> && Broadcastable<A, B>) {
        return combine_to<OP, Commutes, Bool>(y, x);
    } else {
        static_assert(Broadcastable<B, A>, "operands are not broadcastable");
        using R = std::conditional_t<Bool, bool, arith_t<typename A::ValueType, typename B::ValueType>>;
        Tensor<R, Allocator<kCUDA>, typename A::Dims> z;
        auto yb = y.template broadcastTo<typename A::Dims>();
        chain(z, {ins(OP, 1, 0.0, dtype_v<R>)}, x, yb);
        return z;
    }
}

// CombineNode (Kernels.hpp:28-31): x = f(x, broadcast(y)) in place.
template <int OP, AnyTensor A, AnyTensor B>
A& combine_inplace(A& x, const B& y) {
    auto yb = y.template broadcastTo<typename A::Dims>();
    chain(x, {ins(OP, 1, 0.0, dtype_v<typename A::ValueType>)}, x, yb);
    return x;
}

template <int OP, bool Bool, AnyTensor T, Scalar S>
auto with_scalar(const T& t, S s) {
    using R = std::conditional_t<Bool, bool, arith_t<typename T::ValueType, scalar_t<S>>>;
    return unary_new<R>(t, OP, (double)s, TADMA_SRC_IMM);
}

}  // namespace detail

// tensor (op) scalar -- EltwiseNode with the scalar captured (Tensor.hpp:499-510)
template <AnyTensor T, Scalar S> auto operator+(const T& t, S v) { return detail::with_scalar<TADMA_OP_ADD, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator-(const T& t, S v) { return detail::with_scalar<TADMA_OP_SUB, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator*(const T& t, S v) { return detail::with_scalar<TADMA_OP_MUL, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator/(const T& t, S v) { return detail::with_scalar<TADMA_OP_DIV, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator-(S v, const T& t) { return detail::with_scalar<TADMA_OP_RSUB, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator/(S v, const T& t) { return detail::with_scalar<TADMA_OP_RDIV, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator+(S v, const T& t) { return detail::with_scalar<TADMA_OP_ADD, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator*(S v, const T& t) { return detail::with_scalar<TADMA_OP_MUL, false>(t, v); }
template <AnyTensor T, Scalar S> auto operator>(const T& t, S v) { return detail::with_scalar<TADMA_OP_GT, true>(t, v); }
template <AnyTensor T, Scalar S> auto operator<(const T& t, S v) { return detail::with_scalar<TADMA_OP_LT, true>(t, v); }
template <AnyTensor T, Scalar S> auto operator==(const T& t, S v) { return detail::with_scalar<TADMA_OP_EQ, true>(t, v); }
template <AnyTensor T, Scalar S> auto operator!=(const T& t, S v) { return detail::with_scalar<TADMA_OP_NE, true>(t, v); }

// tensor (op) tensor -- CombineToNode (Tensor.hpp:512-533)
template <AnyTensor A, AnyTensor B> auto operator+(const A& a, const B& b) { return detail::combine_to<TADMA_OP_ADD, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator-(const A& a, const B& b) { return detail::combine_to<TADMA_OP_SUB, false, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator*(const A& a, const B& b) { return detail::combine_to<TADMA_OP_MUL, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator/(const A& a, const B& b) { return detail::combine_to<TADMA_OP_DIV, false, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator>(const A& a, const B& b) { return detail::combine_to<TADMA_OP_GT, false, true>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator<(const A& a, const B& b) { return detail::combine_to<TADMA_OP_LT, false, true>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator==(const A& a, const B& b) { return detail::combine_to<TADMA_OP_EQ, true, true>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator!=(const A& a, const B& b) { return detail::combine_to<TADMA_OP_NE, true, true>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator&(const A& a, const B& b) { return detail::combine_to<TADMA_OP_AND, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator|(const A& a, const B& b) { return detail::combine_to<TADMA_OP_OR, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator^(const A& a, const B& b) { return detail::combine_to<TADMA_OP_XOR, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator&&(const A& a, const B& b) { return detail::combine_to<TADMA_OP_LAND, true, true>(a, b); }
template <AnyTensor A, AnyTensor B> auto operator||(const A& a, const B& b) { return detail::combine_to<TADMA_OP_LOR, true, true>(a, b); }
template <AnyTensor T> auto operator-(const T& t) { return detail::unary_new<typename T::ValueType>(t, TADMA_OP_NEG); }

// compound assignment, in place (Tensor.hpp:494-497, 518-521, 535-537)
template <AnyTensor T, Scalar S> T& operator+=(T& t, S v) { detail::unary_inplace(t, TADMA_OP_ADD, (double)v, TADMA_SRC_IMM); return t; }
template <AnyTensor T, Scalar S> T& operator-=(T& t, S v) { detail::unary_inplace(t, TADMA_OP_SUB, (double)v, TADMA_SRC_IMM); return t; }
template <AnyTensor T, Scalar S> T& operator*=(T& t, S v) { detail::unary_inplace(t, TADMA_OP_MUL, (double)v, TADMA_SRC_IMM); return t; }
template <AnyTensor T, Scalar S> T& operator/=(T& t, S v) { detail::unary_inplace(t, TADMA_OP_DIV, (double)v, TADMA_SRC_IMM); return t; }
template <AnyTensor A, AnyTensor B> A& operator+=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_ADD>(a, b); }
template <AnyTensor A, AnyTensor B> A& operator-=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_SUB>(a, b); }
template <AnyTensor A, AnyTensor B> A& operator*=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_MUL>(a, b); }
template <AnyTensor A, AnyTensor B> A& operator/=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_DIV>(a, b); }
template <AnyTensor A, AnyTensor B> A& operator&=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_AND>(a, b); }
template <AnyTensor A, AnyTensor B> A& operator|=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_OR>(a, b); }
template <AnyTensor A, AnyTensor B> A& operator^=(A& a, const B& b) { return detail::combine_inplace<TADMA_OP_XOR>(a, b); }

// MKOP unary ops (Operations.hpp:166-182): Inplace = true overwrites t.
#define TADMA_MKOP(name, OPC, RESULT)                                                    \
    template <bool Inplace = true, AnyTensor T>                                          \
    auto name(T&& t) {                                                                   \
        using TT = std::decay_t<T>;                                                      \
        if constexpr (Inplace) {                                                         \
            detail::unary_inplace(t, OPC);                                               \
            return TT(t);                                                                \
        } else {                                                                         \
            return detail::unary_new<RESULT>(t, OPC);                                    \
        }                                                                                \
    }

TADMA_MKOP(abs, TADMA_OP_ABS, typename TT::ValueType)
TADMA_MKOP(sin, TADMA_OP_SIN, math_t<typename TT::ValueType>)
TADMA_MKOP(cos, TADMA_OP_COS, math_t<typename TT::ValueType>)
TADMA_MKOP(tan, TADMA_OP_TAN, math_t<typename TT::ValueType>)
TADMA_MKOP(asin, TADMA_OP_ASIN, math_t<typename TT::ValueType>)
TADMA_MKOP(acos, TADMA_OP_ACOS, math_t<typename TT::ValueType>)
TADMA_MKOP(atan, TADMA_OP_ATAN, math_t<typename TT::ValueType>)
TADMA_MKOP(asinh, TADMA_OP_ASINH, math_t<typename TT::ValueType>)
TADMA_MKOP(acosh, TADMA_OP_ACOSH, math_t<typename TT::ValueType>)
TADMA_MKOP(atanh, TADMA_OP_ATANH, math_t<typename TT::ValueType>)
TADMA_MKOP(exp, TADMA_OP_EXP, math_t<typename TT::ValueType>)
TADMA_MKOP(log, TADMA_OP_LOG, math_t<typename TT::ValueType>)
TADMA_MKOP(sqrt, TADMA_OP_SQRT, math_t<typename TT::ValueType>)
TADMA_MKOP(erf, TADMA_OP_ERF, math_t<typename TT::ValueType>)
TADMA_MKOP(relu, TADMA_OP_RELU, typename TT::ValueType)
TADMA_MKOP(sigmoid, TADMA_OP_SIGMOID, math_t<typename TT::ValueType>)
TADMA_MKOP(tanh, TADMA_OP_TANH, math_t<typename TT::ValueType>)
TADMA_MKOP(gelu, TADMA_OP_GELU, double)
TADMA_MKOP(negate, TADMA_OP_NEG, typename TT::ValueType)
#undef TADMA_MKOP

// pow (Operations.hpp:186-188); pow(x, 2) is evaluated as x * x.
template <bool Inplace = true, AnyTensor T, Scalar S>
auto pow(T&& t, S s) {
    using TT = std::decay_t<T>;
    if constexpr (Inplace) {
        detail::unary_inplace(t, TADMA_OP_POW, (double)s, TADMA_SRC_IMM);
        return TT(t);
    } else {
        return detail::unary_new<arith_t<math_t<typename TT::ValueType>, scalar_t<S>>>(t, TADMA_OP_POW, (double)s,
                                                                                       TADMA_SRC_IMM);
    }
}

// ---------------------------------------------------------------- reductions --

namespace detail {
template <int D, int Rank>
constexpr int real_dim = D < 0 ? Rank + D : D;

template <int OP, int D, bool KeepDims, typename R, AnyTensor T>
auto reduce_to(const T& t) {
    constexpr int Ax = real_dim<D, T::Rank>;
    static_assert(Ax >= 0 && Ax < T::Rank, "reduction axis out of range");
    using OutDims = std::conditional_t<KeepDims, typename T::Dims::template Set<Ax, 1>, typename T::Dims::template Remove<Ax>>;
    Tensor<R, Allocator<kCUDA>, OutDims> out;
    // A reduction of a deferred element-wise result: one reduce_chain, deferred;
    // a last-axis reduction of anything else: the eager call, deferred, so
    // that the chain that reads it can take it into one row program.
    if (defer_reduce(OP, Ax, out, t)) return out;
    if constexpr (std::is_floating_point_v<R> || std::is_same_v<R, __half> || std::is_same_v<R, __nv_bfloat16>)
        if (defer_plain_reduce(OP, Ax, out, t)) return out;
    tadma_tensor i = t.describe(), o = out.describe();
    check(tadma_b200_reduce(OP, &i, Ax, TADMA_OP_COPY, &o, stream), "tadma reduce");
    return out;
}
}  // namespace detail

template <typename T, typename A, AnySequence D, AnySequence S>
template <int Dm, bool KeepDims>
auto Tensor<T, A, D, S>::sum() const { return detail::reduce_to<TADMA_REDUCE_SUM, Dm, KeepDims, T>(*this); }
template <typename T, typename A, AnySequence D, AnySequence S>
template <int Dm, bool KeepDims>
auto Tensor<T, A, D, S>::min() const { return detail::reduce_to<TADMA_REDUCE_MIN, Dm, KeepDims, T>(*this); }
template <typename T, typename A, AnySequence D, AnySequence S>
template <int Dm, bool KeepDims>
auto Tensor<T, A, D, S>::max() const { return detail::reduce_to<TADMA_REDUCE_MAX, Dm, KeepDims, T>(*this); }
template <typename T, typename A, AnySequence D, AnySequence S>
template <int Dm, bool KeepDims>
auto Tensor<T, A, D, S>::mean() const { return detail::reduce_to<TADMA_REDUCE_MEAN, Dm, KeepDims, T>(*this); }
template <typename T, typename A, AnySequence D, AnySequence S>
template <int Dm, bool KeepDims>
auto Tensor<T, A, D, S>::argmax() const { return detail::reduce_to<TADMA_REDUCE_ARGMAX, Dm, KeepDims, int64_t>(*this); }
template <typename T, typename A, AnySequence D, AnySequence S>
template <int Dm, bool KeepDims>
auto Tensor<T, A, D, S>::argmin() const { return detail::reduce_to<TADMA_REDUCE_ARGMIN, Dm, KeepDims, int64_t>(*this); }

// ------------------------------------------------- fused reduce + broadcast --

// softmax<Dim, Inplace> (Operations.hpp:190-193): one fused pass, max-subtracted.
template <int Dim, bool Inplace = true, AnyTensor T>
auto softmax(T t) {
    constexpr int Ax = detail::real_dim<Dim, T::Rank>;
    if constexpr (Inplace) detail::sync_write_of(t);
    tadma_tensor i = t.describe();
    if constexpr (Inplace) {
        detail::check(tadma_b200_softmax(&i, Ax, &i, stream), "tadma softmax");
        return t;
    } else {
        TensorLike<T> out;
        tadma_tensor o = out.describe();
        detail::check(tadma_b200_softmax(&i, Ax, &o, stream), "tadma softmax");
        return out;
    }
}

namespace detail {
template <AnyTensor G>
tadma_tensor vec_desc(const G& g, int64_t L) {
    static_assert(G::NormalStrides, "gamma / beta must be contiguous");
    if (G::Size != L) throw std::runtime_error("tadma layer_norm: gamma / beta length differs from the normalised axis");
    tadma_tensor d = g.describe();
    d.rank = 1;
    d.dims[0] = L;
    d.strides[0] = 1;
    return d;
}

template <int D, bool Inplace, int Mode, AnyTensor T, AnyTensor G, AnyTensor B>
auto layer_norm_impl(T& t, const G& gamma, const B& beta, double eps) {
    constexpr int Ax = real_dim<D, T::Rank>;
    static_assert(Ax == T::Rank - 1, "layer_norm normalises the last axis");
    if constexpr (Inplace) sync_write_of(t);
    tadma_tensor i = t.describe(), g = vec_desc(gamma, T::Dims::Arr[Ax]), b = vec_desc(beta, T::Dims::Arr[Ax]);
    if constexpr (Inplace) {
        check(tadma_b200_layer_norm(&i, Ax, &g, &b, eps, Mode, &i, stream), "tadma layer_norm");
        return t;
    } else {
        TensorLike<T> out;
        tadma_tensor o = out.describe();
        check(tadma_b200_layer_norm(&i, Ax, &g, &b, eps, Mode, &o, stream), "tadma layer_norm");
        return out;
    }
}
}  // namespace detail

// layer_norm<D, Inplace> (Operations.hpp:205-220): (x - mean) / (std + eps) * gamma + beta
// (the reference adds eps to the population std).
template <int D, bool Inplace = true, AnyTensor T, AnyTensor G, AnyTensor B>
auto layer_norm(T&& t, const G& gamma, const B& beta, float eps = 1e-5f) {
    return detail::layer_norm_impl<D, Inplace, TADMA_LN_TADMA>(t, gamma, beta, eps);
}

// ONNX LayerNormalization: (x - mean) / sqrt(var + eps) * gamma + beta.
template <int D, bool Inplace = true, AnyTensor T, AnyTensor G, AnyTensor B>
auto layer_norm_onnx(T&& t, const G& gamma, const B& beta, float eps = 1e-5f) {
    return detail::layer_norm_impl<D, Inplace, TADMA_LN_ONNX>(t, gamma, beta, eps);
}

// rms_norm<D, Inplace> (Operations.hpp:222-233): x / sqrt(mean(x^2)).
template <int D, bool Inplace = true, AnyTensor T>
auto rms_norm(T&& t) {
    using TT = std::decay_t<T>;
    constexpr int Ax = detail::real_dim<D, TT::Rank>;
    if constexpr (Inplace) detail::sync_write_of(t);
    tadma_tensor i = t.describe();
    if constexpr (Inplace) {
        detail::check(tadma_b200_rms_norm(&i, Ax, 0.0, &i, stream), "tadma rms_norm");
        return TT(t);
    } else {
        TensorLike<TT> out;
        tadma_tensor o = out.describe();
        detail::check(tadma_b200_rms_norm(&i, Ax, 0.0, &o, stream), "tadma rms_norm");
        return out;
    }
}

// mean_stddev<D> (Operations.hpp:195-203): population mean and std, keep-dims.
template <int D, AnyTensor T>
auto mean_stddev(const T& t) {
    auto mean = t.template mean<D>();
    auto centered = t - mean;
    constexpr int Ax = detail::real_dim<D, T::Rank>;
    Tensor<typename decltype(centered)::ValueType, Allocator<kCUDA>, typename T::Dims::template Set<Ax, 1>> stddev;
    tadma_tensor c = centered.describe(), s = stddev.describe();
    detail::check(tadma_b200_reduce(TADMA_REDUCE_RMS, &c, Ax, TADMA_OP_COPY, &s, stream), "tadma mean_stddev");
    return std::pair{mean, stddev};
}

// ------------------------------------------------------------- where / gather --

// where(c, x, y) (Operations.hpp:235-242): result has the condition's dims.
template <AnyTensor Cond, AnyTensor X, AnyTensor Y>
auto where(const Cond& c, const X& x, const Y& y) {
    using R = arith_t<typename X::ValueType, typename Y::ValueType>;
    Tensor<R, Allocator<kCUDA>, typename Cond::Dims> out;
    auto xb = x.template broadcastTo<typename Cond::Dims>();
    auto yb = y.template broadcastTo<typename Cond::Dims>();
    detail::chain(out, {detail::ins(TADMA_OP_WHERE, 1, 0.0, dtype_v<R>, 2)}, c, xb, yb);
    return out;
}

namespace detail {
template <int Axis, AnyTensor In, AnyTensor Idx>
consteval auto gather_dims_arr() {
    std::array<int64_t, In::Rank - 1 + Idx::Rank> a{};
    int k = 0;
    for (int i = 0; i < Axis; i++) a[k++] = In::Dims::Arr[i];
    for (int i = 0; i < Idx::Rank; i++) a[k++] = Idx::Dims::Arr[i];
    for (int i = Axis + 1; i < In::Rank; i++) a[k++] = In::Dims::Arr[i];
    return a;
}
}  // namespace detail

// gather<Axis>(input, indices) (Operations.hpp:244-262): ONNX Gather.  A
// one-element host index tensor gives a view (index<Axis>), as in the reference.
template <int Axis = 0, AnyTensor In, AnyTensor Idx>
auto gather(const In& input, const Idx& indices) {
    constexpr int Ax = detail::real_dim<Axis, In::Rank>;
    if constexpr (Idx::IsScalar && Idx::Rank == 0 && Idx::device == kCPU) {
        return input.template index<Ax>((int64_t)indices.data.view[0]);
    } else {
        using OutDims = SeqFromArray<detail::gather_dims_arr<Ax, In, Idx>()>;
        Tensor<typename In::ValueType, Allocator<kCUDA>, OutDims> out;
        tadma_tensor t = input.describe(), i = indices.describe(), o = out.describe(), none{};
        detail::check(tadma_b200_gather(&t, Ax, &i, &none, &o, stream), "tadma gather");
        return out;
    }
}

// gather<Axis>(input, indices, add): the gather with a fused broadcast add
// (embedding lookup + position table), one kernel.
template <int Axis = 0, AnyTensor In, AnyTensor Idx, AnyTensor Add>
auto gather_add(const In& input, const Idx& indices, const Add& add) {
    constexpr int Ax = detail::real_dim<Axis, In::Rank>;
    using OutDims = SeqFromArray<detail::gather_dims_arr<Ax, In, Idx>()>;
    using R = arith_t<typename In::ValueType, typename Add::ValueType>;
    Tensor<R, Allocator<kCUDA>, OutDims> out;
    auto ab = add.template broadcastTo<OutDims>();
    tadma_tensor t = input.describe(), i = indices.describe(), a = ab.describe(), o = out.describe();
    detail::check(tadma_b200_gather(&t, Ax, &i, &a, &o, stream), "tadma gather");
    return out;
}

// concat<Axis>(t0, t1, ...) (Operations.hpp:265-287): one strided copy per input.
template <int Axis = 0, AnyTensor T, AnyTensor... Ts>
auto concat(const T& t0, const Ts&... ts) {
    constexpr int Ax = detail::real_dim<Axis, T::Rank>;
    static_assert(((Ts::Rank == T::Rank) && ...), "concat needs equal ranks");
    static_assert(((typename T::Dims::template Set<Ax, 0>() == typename Ts::Dims::template Set<Ax, 0>()) && ...),
                  "concat needs equal dims off the axis");
    constexpr int64_t NewSize = T::Dims::Arr[Ax] + (int64_t(0) + ... + Ts::Dims::Arr[Ax]);
    Tensor<typename T::ValueType, Allocator<kCUDA>, typename T::Dims::template Set<Ax, NewSize>> out;
    using OutT = decltype(out);
    int64_t offset = 0;
    auto put = [&](const auto& part) {
        using P = std::decay_t<decltype(part)>;
        Tensor<typename T::ValueType, Allocator<kCUDA>, typename P::Dims, typename OutT::Strides> dst(
            out.data + offset * OutT::Strides::Arr[Ax]);
        detail::chain(dst, {detail::ins(TADMA_OP_COPY)}, part);
        offset += P::Dims::Arr[Ax];
    };
    put(t0);
    (put(ts), ...);
    return out;
}

// ----------------------------------------------------------- fused chains --

// tadma::fused<R>(x, steps...): a linear chain of up to 16 ops in ONE kernel,
// e.g. fused<__nv_bfloat16>(x, fuse::mul(0.5), fuse::add(bias), fuse::gelu())
// computes gelu(x * 0.5 + bias) in fp32 registers and writes bf16 once: the
// fused form of the reference's tape merge (MergeNodes, Node.hpp:189-224)
// without materialising the intermediates.  Tensor operands (at most 3)
// broadcast to x's dims.
namespace fuse {
struct Imm {
    int op;
    double v;
};
struct Un {
    int op;
};
template <AnyTensor T>
struct Ten {
    int op;
    const T* t;
};
#define TADMA_FUSE_BIN(name, OPC)                                       \
    inline Imm name(double v) { return {OPC, v}; }                      \
    template <AnyTensor T>                                              \
    Ten<T> name(const T& t) { return {OPC, &t}; }
TADMA_FUSE_BIN(add, TADMA_OP_ADD)
TADMA_FUSE_BIN(sub, TADMA_OP_SUB)
TADMA_FUSE_BIN(mul, TADMA_OP_MUL)
TADMA_FUSE_BIN(div, TADMA_OP_DIV)
TADMA_FUSE_BIN(rsub, TADMA_OP_RSUB)
TADMA_FUSE_BIN(rdiv, TADMA_OP_RDIV)
TADMA_FUSE_BIN(maximum, TADMA_OP_MAX)
TADMA_FUSE_BIN(minimum, TADMA_OP_MIN)
TADMA_FUSE_BIN(pow, TADMA_OP_POW)
#undef TADMA_FUSE_BIN
inline Un exp() { return {TADMA_OP_EXP}; }
inline Un log() { return {TADMA_OP_LOG}; }
inline Un sqrt() { return {TADMA_OP_SQRT}; }
inline Un erf() { return {TADMA_OP_ERF}; }
inline Un relu() { return {TADMA_OP_RELU}; }
inline Un sigmoid() { return {TADMA_OP_SIGMOID}; }
inline Un tanh() { return {TADMA_OP_TANH}; }
inline Un gelu() { return {TADMA_OP_GELU}; }
inline Un neg() { return {TADMA_OP_NEG}; }
inline Un abs() { return {TADMA_OP_ABS}; }
}  // namespace fuse

namespace detail {
template <AnyTensor X>
struct FuseBuilder {
    std::array<tadma_instr, TADMA_MAX_INSTR> prog{};
    std::array<tadma_tensor, TADMA_MAX_INPUTS> ins{};
    int n_instr = 0, n_ins = 1;
    void push(const fuse::Imm& s) { prog.at(n_instr++) = detail::ins(s.op, TADMA_SRC_IMM, s.v); }
    void push(const fuse::Un& s) { prog.at(n_instr++) = detail::ins(s.op); }
    template <AnyTensor T>
    void push(const fuse::Ten<T>& s) {
        if (n_ins >= TADMA_MAX_INPUTS) throw std::runtime_error("tadma fused: at most 5 tensor operands");
        ins[n_ins] = s.t->template broadcastTo<typename X::Dims>().describe();
        prog.at(n_instr++) = detail::ins(s.op, n_ins++);
    }
};
}  // namespace detail

template <Element R, AnyTensor X, typename... Steps>
auto fused(const X& x, const Steps&... steps) {
    static_assert(sizeof...(Steps) <= TADMA_MAX_INSTR, "at most 16 fused ops");
    detail::FuseBuilder<X> b;
    b.ins[0] = x.describe();
    (b.push(steps), ...);
    Tensor<R, Allocator<kCUDA>, typename X::Dims> out;
    tadma_tensor o = out.describe();
    detail::check(tadma_b200_eltwise(&o, b.ins.data(), b.n_ins, b.prog.data(), b.n_instr, TADMA_COMPUTE_F32, stream),
                  "tadma fused");
    return out;
}


// tadma::fused_reduce<OP, Axis, KeepDims>(x, steps...): the chain of
// tadma::fused reduced along Axis in the same kernel (tadma_b200_reduce_chain),
// e.g. fused_reduce<TADMA_REDUCE_SUM, -1, false>(A, fuse::add(b), fuse::exp())
// for sum<-1>(exp(A + b)); the chain's values never reach HBM.  The result
// is fp32 (int64 for ARGMAX / ARGMIN).
template <int OP, int Axis, bool KeepDims = true, AnyTensor X, typename... Steps>
auto fused_reduce(const X& x, const Steps&... steps) {
    static_assert(sizeof...(Steps) <= TADMA_MAX_INSTR, "at most 16 fused ops");
    constexpr int Ax = detail::real_dim<Axis, X::Rank>;
    static_assert(Ax >= 0 && Ax < X::Rank, "reduction axis out of range");
    detail::FuseBuilder<X> b;
    b.ins[0] = x.describe();
    (b.push(steps), ...);
    using OutDims = std::conditional_t<KeepDims, typename X::Dims::template Set<Ax, 1>, typename X::Dims::template Remove<Ax>>;
    using R = std::conditional_t<OP == TADMA_REDUCE_ARGMAX || OP == TADMA_REDUCE_ARGMIN, int64_t, float>;
    Tensor<R, Allocator<kCUDA>, OutDims> out;
    tadma_tensor o = out.describe();
    detail::check(tadma_b200_reduce_chain(OP, b.ins.data(), b.n_ins, b.prog.data(), b.n_instr, TADMA_COMPUTE_F32, Ax,
                                          &o, stream),
                  "tadma fused_reduce");
    return out;
}

}  // namespace tadma
