// Lazy.hpp - deferred element-wise chains: the reference's tape merge
// (ExecutionTape::Append / FindMergeable / Optimize / Evaluate,
// ExecutionTape.hpp:41-192, and MergeNodes, Node.hpp:189-224) as expression
// values that fuse into the consumer's kernel.
//
// tadma::lazy(x) wraps a CUDA tensor.  The element-wise operators (+ - * /
// with a scalar or a tensor, comparisons, bitwise and logical ops, compound
// assignment) and the unary functions (exp, tanh, gelu, pow, ...) applied to
// a lazy value record one instruction of a chain instead of launching a
// kernel.  Each instruction rounds to the element type that the eager call
// would have produced and is computed in the precision the eager call would
// have used, so a chain gives the same bits as the same calls made eagerly.
// The chain runs as ONE kernel where it is consumed:
// * .eval(), or conversion to its Tensor type: tadma_b200_eltwise into a new
//   tensor;
// * .sum / .min / .max / .mean / .argmax / .argmin<D, KeepDims>():
//   tadma_b200_reduce_chain; the chain's values never reach HBM (equal to the
//   eager reduction bit for bit for min / max / argmax / argmin, sums within
//   the fp32 reduction tolerance);
// * any other call that takes a tensor (softmax, layer_norm, gather, an
//   eager operator with a lazy operand): a lazy value satisfies AnyTensor, and
//   its describe() materialises it once and keeps the result.
// A chain holds at most 16 instructions and 5 tensors besides its source,
// each broadcast to the source's dims.  An instruction that would exceed
// either limit, or that the eager call would compute in another precision
// than the chain's (a double result after float ones, an integer op after
// float ones), first materialises the chain and starts a new one from it.
// Unlike the eager in-place variants (Inplace = true), a lazy chain never
// writes its operands; the Inplace flag only selects the result type.
#pragma once

#include <memory>

#include "Operations.hpp"

namespace tadma {

template <typename R, AnySequence Dims_>
struct Lazy;

namespace detail {

template <typename X>
struct is_lazy : std::false_type {};
template <typename R, typename D>
struct is_lazy<Lazy<R, D>> : std::true_type {};

// dtype_float, dtype_wide, op_transcendental, eager_compute and same_view
// are shared with the deferred evaluation (Deferred.hpp).

// The recorded chain: operands (ins[0] is the source), instructions, the
// chain's precision (AUTO until the first instruction fixes it) and shared
// ownership of every operand's storage.
struct LazyChain {
    std::array<tadma_instr, TADMA_MAX_INSTR> prog{};
    std::array<tadma_tensor, TADMA_MAX_INPUTS> ins{};
    std::array<std::shared_ptr<const void>, TADMA_MAX_INPUTS> keep{};
    int n_instr = 0, n_ins = 1, compute = TADMA_COMPUTE_AUTO;
};

// Index of the operand of `c` that is the same view as `t`, or -1.
inline int find_operand(const LazyChain& c, const tadma_tensor& t) {
    for (int k = 0; k < c.n_ins; k++)
        if (same_view(c.ins[k], t)) return k;
    return -1;
}

// Swapped operand order for `tensor (op) lazy`: acc is the lazy value.
constexpr int reversed_op(int op) {
    switch (op) {
    case TADMA_OP_SUB: return TADMA_OP_RSUB;
    case TADMA_OP_DIV: return TADMA_OP_RDIV;
    case TADMA_OP_GT: return TADMA_OP_LT;
    case TADMA_OP_LT: return TADMA_OP_GT;
    case TADMA_OP_GE: return TADMA_OP_LE;
    case TADMA_OP_LE: return TADMA_OP_GE;
    default: return op;  // + * == != & | ^ && || commute
    }
}

}  // namespace detail

template <typename T>
concept LazyTensor = AnyTensor<T> && detail::is_lazy<std::decay_t<T>>::value;
template <typename A, typename B>
concept LazyOperand = LazyTensor<A> || LazyTensor<B>;

template <typename R, AnySequence Dims_>
struct Lazy {
    using ValueType = R;
    using Dims = Dims_;
    using Allocator = tadma::Allocator<kCUDA>;
    using AllocatorType = Allocator;
    using Strides = DefaultStrides<Dims>;
    static constexpr Memory device = kCUDA;
    static constexpr int64_t Rank = Dims::Size;
    static constexpr int64_t Size = Dims::Product();
    using Result = Tensor<R, Allocator, Dims>;

    detail::LazyChain chain;
    mutable std::shared_ptr<Result> cache;  // filled by describe()

    static consteval int64_t Dim(int i) { return Dims::Values(i < 0 ? i + Rank : i); }

    // Runs the chain into a new tensor (one kernel).  After describe() has
    // materialised the value, the value IS that tensor (an in-place call on it,
    // e.g. softmax<D, true>, writes there): eval() returns it, and new steps
    // and reductions start from it.
    Result eval() const {
        if (cache) return *cache;
        Result out;
        tadma_tensor o = out.describe();
        detail::check(tadma_b200_eltwise(&o, chain.ins.data(), chain.n_ins, chain.prog.data(), chain.n_instr,
                                         chain.compute, stream),
                      "tadma lazy eval");
        return out;
    }
    operator Result() const { return eval(); }
    Result contiguous() const { return eval(); }

    // The materialised value, computed once per lazy value.
    const Result& materialised() const {
        if (!cache) cache = std::make_shared<Result>(eval());
        return *cache;
    }
    tadma_tensor describe() const { return materialised().describe(); }

    template <AnySequence TargetDims>
    auto broadcastTo() const { return materialised().template broadcastTo<TargetDims>(); }
    template <AnyTensor U>
    auto broadcastTo() const { return materialised().template broadcastTo<U>(); }
    template <AnyTensor U>
    auto broadcastTo(const U& u) const { return materialised().broadcastTo(u); }
    template <int... P>
    auto transpose() const { return materialised().template transpose<P...>(); }
    template <AnySequence NewDims>
    auto reshape() const { return materialised().template reshape<NewDims>(); }
    template <auto... NewDims>
    auto reshape() const { return materialised().template reshape<NewDims...>(); }

    // Appends `op` with result type R2.  `b` is TADMA_SRC_IMM (imm) or
    // TADMA_SRC_NONE; each given operand (a view of this chain's dims) takes
    // the place of b, then c (TADMA_OP_WHERE reads both).  An operand the
    // chain already reads (the same view) is not added twice.
    struct Operand {
        tadma_tensor desc;
        std::shared_ptr<const void> keep;
    };
    template <typename R2>
    Lazy<R2, Dims> then(int op, int b, double imm, const Operand* ob = nullptr, const Operand* oc = nullptr) const {
        detail::LazyChain cur = current();
        const int cm = detail::eager_compute(dtype_v<R2>, dtype_v<R>, ob ? ob->desc.dtype : -1, op,
                                             b == TADMA_SRC_IMM, imm, oc ? oc->desc.dtype : -1);
        int fresh = 0;  // operand slots this step adds
        if (ob && detail::find_operand(cur, ob->desc) < 0) fresh++;
        if (oc && detail::find_operand(cur, oc->desc) < 0 && !(ob && detail::same_view(ob->desc, oc->desc))) fresh++;
        const bool fits = cur.n_instr < TADMA_MAX_INSTR && cur.n_ins + fresh <= TADMA_MAX_INPUTS &&
                          (cur.compute == TADMA_COMPUTE_AUTO || cur.compute == cm);
        Lazy<R2, Dims> next;
        next.chain = fits ? std::move(cur) : restart().chain;
        detail::LazyChain& ch = next.chain;
        auto slot = [&ch](const Operand& o) {
            int k = detail::find_operand(ch, o.desc);
            if (k < 0) {
                k = ch.n_ins++;
                ch.ins[k] = o.desc;
                ch.keep[k] = o.keep;
            }
            return k;
        };
        const int sb = ob ? slot(*ob) : b;
        const int sc = oc ? slot(*oc) : TADMA_SRC_NONE;
        ch.prog[ch.n_instr++] = detail::ins(op, sb, imm, dtype_v<R2>, sc);
        ch.compute = cm;
        return next;
    }
    // The operand view of tensor y broadcast to this chain's dims.
    template <AnyTensor B>
    Operand operand(const B& y) const {
        if constexpr (LazyTensor<B>) {
            return operand(y.materialised());
        } else {
            auto yb = std::make_shared<const decltype(y.template broadcastTo<Dims>())>(y.template broadcastTo<Dims>());
            return Operand{yb->describe(), std::move(yb)};
        }
    }
    template <typename R2, AnyTensor B>
    Lazy<R2, Dims> then(int op, const B& y) const {
        const Operand o = operand(y);
        return then<R2>(op, TADMA_SRC_NONE, 0.0, &o);
    }

    // A chain whose source is this chain's materialised value.
    Lazy restart() const;
    // The chain that new steps extend: this one, or once materialised, a
    // chain over the materialised tensor.
    detail::LazyChain current() const;

    // -------------------------------------------------------- reductions --
    template <int OP, int D, bool KeepDims, typename Out>
    auto reduce() const {
        constexpr int Ax = detail::real_dim<D, Rank>;
        static_assert(Ax >= 0 && Ax < Rank, "reduction axis out of range");
        using OutDims = std::conditional_t<KeepDims, typename Dims::template Set<Ax, 1>, typename Dims::template Remove<Ax>>;
        Tensor<Out, Allocator, OutDims> out;
        tadma_tensor o = out.describe();
        const detail::LazyChain c = current();
        detail::check(tadma_b200_reduce_chain(OP, c.ins.data(), c.n_ins, c.prog.data(), c.n_instr, c.compute, Ax, &o,
                                              stream),
                      "tadma lazy reduce");
        return out;
    }
    template <int D, bool KeepDims = true>
    auto sum() const { return reduce<TADMA_REDUCE_SUM, D, KeepDims, R>(); }
    template <int D, bool KeepDims = true>
    auto min() const { return reduce<TADMA_REDUCE_MIN, D, KeepDims, R>(); }
    template <int D, bool KeepDims = true>
    auto max() const { return reduce<TADMA_REDUCE_MAX, D, KeepDims, R>(); }
    template <int D, bool KeepDims = true>
    auto mean() const { return reduce<TADMA_REDUCE_MEAN, D, KeepDims, R>(); }
    template <int D, bool KeepDims = false>
    auto argmax() const { return reduce<TADMA_REDUCE_ARGMAX, D, KeepDims, int64_t>(); }
    template <int D, bool KeepDims = false>
    auto argmin() const { return reduce<TADMA_REDUCE_ARGMIN, D, KeepDims, int64_t>(); }

    // Casts (to<U>, Tensor.hpp:189-233): a rounding step of the chain.
    template <Element U>
    Lazy<U, Dims> to() const { return then<U>(TADMA_OP_COPY, TADMA_SRC_NONE, 0.0); }
};

// Starts a chain over tensor x (no kernel is launched).
template <AnyCudaTensor X>
    requires(!LazyTensor<X>)
auto lazy(const X& x) {
    using T = typename std::decay_t<X>::ValueType;
    Lazy<T, typename std::decay_t<X>::Dims> l;
    auto keep = std::make_shared<const std::decay_t<X>>(x);
    l.chain.ins[0] = keep->describe();
    l.chain.keep[0] = std::move(keep);
    return l;
}
template <LazyTensor X>
auto lazy(const X& x) {
    return std::decay_t<X>(x);
}

template <typename R, AnySequence D>
Lazy<R, D> Lazy<R, D>::restart() const {
    return lazy(eval());
}
template <typename R, AnySequence D>
detail::LazyChain Lazy<R, D>::current() const {
    return cache ? lazy(*cache).chain : chain;
}

namespace detail {

template <int OP, bool Commutes, bool Bool, AnyTensor A, AnyTensor B>
auto lazy_combine(const A& a, const B& b) {
    if constexpr (LazyTensor<A> && LazyTensor<B>) {
        // Two chains: the right one is materialised and joins the left one as
        // an operand (the interpreter keeps one accumulator).
        return lazy_combine<OP, Commutes, Bool>(a, b.materialised());
    } else if constexpr (LazyTensor<A>) {
        using R = std::conditional_t<Bool, bool, arith_t<typename A::ValueType, typename B::ValueType>>;
        if constexpr (Broadcastable<B, A>) return a.template then<R>(OP, b);
        else return combine_to<OP, Commutes, Bool>(a.materialised(), b);  // the eager rule (swap or error)
    } else {
        // tensor (op) lazy: the result has the tensor's dims (CombineToNode).
        using R = std::conditional_t<Bool, bool, arith_t<typename A::ValueType, typename B::ValueType>>;
        if constexpr (std::is_same_v<typename A::Dims, typename B::Dims>)
            return b.template then<R>(reversed_op(OP), a);
        else if constexpr (Commutes && !Broadcastable<B, A> && Broadcastable<A, B>)
            return b.template then<R>(OP, a);  // the eager swap: b's dims lead
        else return combine_to<OP, Commutes, Bool>(a, b.materialised());
    }
}

template <int OP, bool Bool, LazyTensor L, Scalar S>
auto lazy_scalar(const L& l, S v) {
    using R = std::conditional_t<Bool, bool, arith_t<typename L::ValueType, scalar_t<S>>>;
    return l.template then<R>(OP, TADMA_SRC_IMM, (double)v);
}

}  // namespace detail

// lazy (op) scalar, scalar (op) lazy
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator+(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_ADD, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator-(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_SUB, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator*(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_MUL, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator/(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_DIV, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator-(S v, const T& t) { return detail::lazy_scalar<TADMA_OP_RSUB, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator/(S v, const T& t) { return detail::lazy_scalar<TADMA_OP_RDIV, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator+(S v, const T& t) { return detail::lazy_scalar<TADMA_OP_ADD, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator*(S v, const T& t) { return detail::lazy_scalar<TADMA_OP_MUL, false>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator>(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_GT, true>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator<(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_LT, true>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator==(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_EQ, true>(t, v); }
template <AnyTensor T, Scalar S> requires LazyTensor<T> auto operator!=(const T& t, S v) { return detail::lazy_scalar<TADMA_OP_NE, true>(t, v); }

// lazy (op) tensor, tensor (op) lazy, lazy (op) lazy
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator+(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_ADD, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator-(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_SUB, false, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator*(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_MUL, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator/(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_DIV, false, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator>(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_GT, false, true>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator<(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_LT, false, true>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator==(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_EQ, true, true>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator!=(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_NE, true, true>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator&(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_AND, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator|(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_OR, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator^(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_XOR, true, false>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator&&(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_LAND, true, true>(a, b); }
template <AnyTensor A, AnyTensor B> requires LazyOperand<A, B> auto operator||(const A& a, const B& b) { return detail::lazy_combine<TADMA_OP_LOR, true, true>(a, b); }
template <AnyTensor T> requires LazyTensor<T> auto operator-(const T& t) { return t.template then<typename T::ValueType>(TADMA_OP_NEG, TADMA_SRC_NONE, 0.0); }

// compound assignment on a lazy value: one more step of its chain (the type,
// hence the rounding, stays the lazy value's own).
#define TADMA_LAZY_ASSIGN(sym, OPC)                                                                  \
    template <AnyTensor T, Scalar S>                                                                 \
        requires LazyTensor<T>                                                                       \
    T& operator sym(T& t, S v) {                                                                     \
        t = t.template then<typename T::ValueType>(OPC, TADMA_SRC_IMM, (double)v);                   \
        return t;                                                                                    \
    }                                                                                                \
    template <AnyTensor A, AnyTensor B>                                                              \
        requires LazyTensor<A>                                                                       \
    A& operator sym(A& a, const B& b) {                                                              \
        a = a.template then<typename A::ValueType>(OPC, b);                                          \
        return a;                                                                                    \
    }
TADMA_LAZY_ASSIGN(+=, TADMA_OP_ADD)
TADMA_LAZY_ASSIGN(-=, TADMA_OP_SUB)
TADMA_LAZY_ASSIGN(*=, TADMA_OP_MUL)
TADMA_LAZY_ASSIGN(/=, TADMA_OP_DIV)
#undef TADMA_LAZY_ASSIGN

// MKOP unary ops on a lazy value: Inplace keeps the value's type (the eager
// in-place call rounds into the input's buffer), Inplace = false takes the
// eager result type (Operations.hpp:166-182).
#define TADMA_LAZY_MKOP(name, OPC, RESULT)                                                \
    template <bool Inplace = true, AnyTensor T>                                           \
        requires LazyTensor<T>                                                            \
    auto name(T&& t) {                                                                    \
        using TT = std::decay_t<T>;                                                       \
        using R2 = std::conditional_t<Inplace, typename TT::ValueType, RESULT>;           \
        return t.template then<R2>(OPC, TADMA_SRC_NONE, 0.0);                             \
    }
TADMA_LAZY_MKOP(abs, TADMA_OP_ABS, typename TT::ValueType)
TADMA_LAZY_MKOP(sin, TADMA_OP_SIN, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(cos, TADMA_OP_COS, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(tan, TADMA_OP_TAN, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(asin, TADMA_OP_ASIN, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(acos, TADMA_OP_ACOS, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(atan, TADMA_OP_ATAN, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(asinh, TADMA_OP_ASINH, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(acosh, TADMA_OP_ACOSH, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(atanh, TADMA_OP_ATANH, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(exp, TADMA_OP_EXP, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(log, TADMA_OP_LOG, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(sqrt, TADMA_OP_SQRT, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(erf, TADMA_OP_ERF, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(relu, TADMA_OP_RELU, typename TT::ValueType)
TADMA_LAZY_MKOP(sigmoid, TADMA_OP_SIGMOID, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(tanh, TADMA_OP_TANH, math_t<typename TT::ValueType>)
TADMA_LAZY_MKOP(gelu, TADMA_OP_GELU, double)
TADMA_LAZY_MKOP(negate, TADMA_OP_NEG, typename TT::ValueType)
#undef TADMA_LAZY_MKOP

// where(c, x, y) with a lazy condition (Operations.hpp:235-242): one
// TADMA_OP_WHERE step reading x and y as operands; the result has the
// condition's dims and the eager result type.
template <AnyTensor Cond, AnyTensor X, AnyTensor Y>
    requires LazyTensor<Cond>
auto where(const Cond& c, const X& x, const Y& y) {
    using R = arith_t<typename X::ValueType, typename Y::ValueType>;
    const auto ox = c.operand(x), oy = c.operand(y);
    return c.template then<R>(TADMA_OP_WHERE, TADMA_SRC_NONE, 0.0, &ox, &oy);
}

template <bool Inplace = true, AnyTensor T, Scalar S>
    requires LazyTensor<T>
auto pow(T&& t, S s) {
    using TT = std::decay_t<T>;
    using R2 = std::conditional_t<Inplace, typename TT::ValueType, arith_t<math_t<typename TT::ValueType>, scalar_t<S>>>;
    return t.template then<R2>(TADMA_OP_POW, TADMA_SRC_IMM, (double)s);
}

}  // namespace tadma
