// Constexpr.hpp - compile-time values of generated graph code.
//
// The ONNX-to-C++ generator (scripts/cppgen.py:100, 123-135 of the
// reference) emits graph constants as types, not tensors:
//   static constexpr ConstexprHolder<1> c = {};                   // a scalar Constant
//   Tensor<T, ConstexprAllocator<Sequence<0, 1, ...>>, Sequence<512>> ids = {};
//                                                                  // a constant tensor
//   auto s = shape(x);                                             // Shape of a static tensor
// and the shape arithmetic of the graph (Gather on a shape, Unsqueeze, Concat,
// Mul / Equal / Where on shape values, Reshape by a computed shape) runs on
// those values.  The reference library never defines these names; here they
// fold at compile time:
// * ConstexprHolder<V>: an empty object whose type carries V.  It converts to
//   V's type in constant expressions, so it can be a template argument
//   (slice<c0, c1>(), unsqueeze<c>()), and arithmetic on two holders gives a
//   holder.
// * ConstTensor<T, Sequence<v...>>: a compile-time 1-D integer tensor (the
//   result of shape(), unsqueeze, concat, gather with a tensor of indices).
//   With one value it converts to T, like a scalar.
// * ConstexprAllocator<Sequence<v...>>: the allocator of a constant device
//   tensor; allocating it uploads the values once, after which the tensor is
//   an ordinary device tensor (views, gather ids, kernels).
// * Tensor::reshape<shape>() (Tensor.hpp) takes a holder (-1 flattens) or a
//   ConstTensor (ONNX Reshape: 0 copies the input dim, one -1 is inferred).
#pragma once

#include <ostream>
#include <type_traits>

#include "Tensor.hpp"

#ifndef TYPE
#define TYPE(x) std::decay_t<decltype(x)>
#endif

namespace tadma {

template <auto V>
struct ConstexprHolder {
    using ValueType = decltype(V);
    static constexpr ValueType value = V;
    constexpr operator ValueType() const { return V; }
    // Unsqueeze of a scalar: a 1-D tensor of one value.
    template <auto Axis = 0>
    constexpr auto unsqueeze() const;
};

template <typename T, AnySequence Values>
struct ConstTensor {
    using ValueType = T;
    using Vals = Values;
    static constexpr int64_t Size = Values::Size;
    static constexpr int64_t Rank = 1;
    static constexpr T at(int64_t i) { return static_cast<T>(Values::Arr[i < 0 ? i + Size : i]); }
    constexpr operator T() const
        requires(Values::Size == 1)
    {
        return at(0);
    }
};

template <auto V>
template <auto Axis>
constexpr auto ConstexprHolder<V>::unsqueeze() const {
    static_assert(std::is_integral_v<decltype(V)>, "unsqueeze of a non-integer constant");
    static_assert(static_cast<int64_t>(Axis) == 0 || static_cast<int64_t>(Axis) == -1, "a scalar unsqueezes on axis 0");
    return ConstTensor<decltype(V), Sequence<static_cast<int64_t>(V)>>{};
}

namespace detail {
template <typename X>
struct is_holder : std::false_type {};
template <auto V>
struct is_holder<ConstexprHolder<V>> : std::true_type {};
template <typename X>
struct is_const_tensor : std::false_type {};
template <typename T, typename S>
struct is_const_tensor<ConstTensor<T, S>> : std::true_type {};
}  // namespace detail

template <typename X>
concept ConstScalar = detail::is_holder<std::decay_t<X>>::value;
template <typename X>
concept ConstVector = detail::is_const_tensor<std::decay_t<X>>::value;
template <typename X>
concept ConstValue = ConstScalar<X> || ConstVector<X>;

namespace detail {
// Values of a compile-time value as an int64 array (a scalar is one value).
template <ConstValue X>
consteval auto const_values() {
    using D = std::decay_t<X>;
    if constexpr (ConstScalar<D>) return std::array<int64_t, 1>{static_cast<int64_t>(D::value)};
    else return D::Vals::Arr;
}
template <typename A, typename B>
consteval std::size_t bcast_size() {
    constexpr auto a = const_values<A>();
    constexpr auto b = const_values<B>();
    static_assert(a.size() == b.size() || a.size() == 1 || b.size() == 1, "shape values do not broadcast");
    return a.size() > b.size() ? a.size() : b.size();
}
template <int OP, typename A, typename B>
consteval auto const_binary() {
    constexpr auto a = const_values<A>();
    constexpr auto b = const_values<B>();
    std::array<int64_t, bcast_size<A, B>()> r{};
    for (std::size_t i = 0; i < r.size(); i++) {
        const int64_t x = a[a.size() == 1 ? 0 : i], y = b[b.size() == 1 ? 0 : i];
        r[i] = OP == 0 ? x + y : OP == 1 ? x - y : OP == 2 ? x * y : OP == 3 ? x / y : int64_t(x == y);
    }
    return r;
}
template <int OP, typename A, typename B>
constexpr auto const_op() {
    if constexpr (ConstScalar<A> && ConstScalar<B>) {
        constexpr auto a = std::decay_t<A>::value;
        constexpr auto b = std::decay_t<B>::value;
        if constexpr (OP == 0) return ConstexprHolder<a + b>{};
        else if constexpr (OP == 1) return ConstexprHolder<a - b>{};
        else if constexpr (OP == 2) return ConstexprHolder<a * b>{};
        else if constexpr (OP == 3) return ConstexprHolder<a / b>{};
        else return ConstexprHolder<a == b>{};
    } else {
        using T = std::conditional_t<OP == 4, bool, int64_t>;
        return ConstTensor<T, SeqFromArray<const_binary<OP, A, B>()>>{};
    }
}
}  // namespace detail

// Shape arithmetic of the graph (Add / Sub / Mul / Div / Equal on constants),
// one holder or constant tensor on each side, folded at compile time.
template <ConstValue A, ConstValue B> constexpr auto operator+(A, B) { return detail::const_op<0, A, B>(); }
template <ConstValue A, ConstValue B> constexpr auto operator-(A, B) { return detail::const_op<1, A, B>(); }
template <ConstValue A, ConstValue B> constexpr auto operator*(A, B) { return detail::const_op<2, A, B>(); }
template <ConstValue A, ConstValue B> constexpr auto operator/(A, B) { return detail::const_op<3, A, B>(); }
template <ConstValue A, ConstValue B> constexpr auto operator==(A, B) { return detail::const_op<4, A, B>(); }

// ONNX Shape of a static tensor: its dims as a 1-D int64 constant.
template <AnyTensor X>
constexpr auto shape(const X&) {
    return ConstTensor<int64_t, typename std::decay_t<X>::Dims>{};
}
// The reference's spelling of the same thing (tfs = "tensor from sequence",
// Tensor.hpp:489-492).
template <AnySequence S>
constexpr auto tfs() {
    return ConstTensor<int64_t, S>{};
}

// ONNX Gather on a constant: a scalar index gives a scalar, a constant
// tensor of indices gives a constant tensor (negative indices count from the end).
template <ConstVector Data, ConstScalar Index>
constexpr auto gather(Data, Index) {
    using D = std::decay_t<Data>;
    constexpr int64_t i = static_cast<int64_t>(std::decay_t<Index>::value);
    static_assert(i >= -D::Size && i < D::Size, "gather index out of range");
    return ConstexprHolder<D::at(i)>{};
}
template <ConstVector Data, ConstVector Index>
constexpr auto gather(Data, Index) {
    using D = std::decay_t<Data>;
    using I = std::decay_t<Index>;
    constexpr auto vals = [] {
        std::array<int64_t, I::Size> r{};
        for (int64_t k = 0; k < I::Size; k++) r[k] = static_cast<int64_t>(D::at(I::at(k)));
        return r;
    }();
    return ConstTensor<typename D::ValueType, SeqFromArray<vals>>{};
}

// ONNX Concat of constants along axis 0 (a scalar counts as one value).
template <int Axis = 0, ConstValue P, ConstValue... Ps>
constexpr auto concat(P, Ps...) {
    static_assert(Axis == 0 || Axis == -1, "constants are 1-D: concat on axis 0");
    constexpr auto vals = [] {
        constexpr std::size_t n = detail::const_values<P>().size() + (std::size_t(0) + ... + detail::const_values<Ps>().size());
        std::array<int64_t, n> r{};
        std::size_t k = 0;
        for (auto v : detail::const_values<P>()) r[k++] = v;
        ((([&] {
             for (auto v : detail::const_values<Ps>()) r[k++] = v;
         })()),
         ...);
        return r;
    }();
    return ConstTensor<int64_t, SeqFromArray<vals>>{};
}

// ONNX Where on constants.
template <ConstValue C, ConstValue X, ConstValue Y>
constexpr auto where(C, X, Y) {
    constexpr auto vals = [] {
        constexpr auto c = detail::const_values<C>();
        constexpr auto x = detail::const_values<X>();
        constexpr auto y = detail::const_values<Y>();
        constexpr std::size_t n = c.size() > x.size() ? (c.size() > y.size() ? c.size() : y.size())
                                                      : (x.size() > y.size() ? x.size() : y.size());
        std::array<int64_t, n> r{};
        for (std::size_t i = 0; i < n; i++)
            r[i] = c[c.size() == 1 ? 0 : i] ? x[x.size() == 1 ? 0 : i] : y[y.size() == 1 ? 0 : i];
        return r;
    }();
    return ConstTensor<int64_t, SeqFromArray<vals>>{};
}

template <auto V>
std::ostream& operator<<(std::ostream& os, ConstexprHolder<V>) {
    return os << V;
}
template <typename T, typename S>
std::ostream& operator<<(std::ostream& os, ConstTensor<T, S>) {
    os << "[";
    for (int64_t i = 0; i < S::Size; i++) os << (i ? ", " : "") << ConstTensor<T, S>::at(i);
    return os << "]";
}

// Allocator of a constant device tensor: allocating uploads Values once.
template <AnySequence Values>
struct ConstexprAllocator;
template <auto... Vs>
struct ConstexprAllocator<Sequence<Vs...>> {
    static constexpr Memory device = kCUDA;
    template <typename T, int64_t Count>
    static HeapStorage<T> allocate() {
        static_assert(Count == sizeof...(Vs), "constant tensor: dims must cover the values");
        static const T host[sizeof...(Vs) > 0 ? sizeof...(Vs) : 1] = {static_cast<T>(Vs)...};
        HeapStorage<T> s = Allocator<kCUDA>::template allocate<T, Count>();
        if constexpr (Count > 0)
            check_cuda(cudaMemcpyAsync(s.view, host, sizeof(T) * Count, cudaMemcpyHostToDevice, stream));
        return s;
    }
};

}  // namespace tadma
