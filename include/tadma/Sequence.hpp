// Sequence.hpp - compile-time integer lists (dims / strides) for the static-shape Tensor API.
//
// Same public surface as the reference's Sequence (include/tadma/Sequence.hpp:6-177):
// Size, Product, Sum, Append, Prepend, Values<I>() / Values(i), Swap, First,
// Last, Merge, Remove, Insert, Set, IndexOf, ContainsOrderedSubset, IsSorted,
// operator==, Array, Apply.  Written in C++20 (nvcc 12.9 has no C++23, so no
// deducing-this and no pack indexing): every derived sequence is computed as a
// constexpr std::array and turned back into a Sequence by SeqFromArray.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <type_traits>
#include <utility>

namespace tadma {

template <auto... Is>
struct Sequence;

namespace detail {
template <auto Arr, typename Idx = std::make_index_sequence<Arr.size()>>
struct SeqFromArrayImpl;
template <auto Arr, std::size_t... I>
struct SeqFromArrayImpl<Arr, std::index_sequence<I...>> {
    using type = Sequence<Arr[I]...>;
};
}  // namespace detail

// Sequence<Arr[0], Arr[1], ...> for a constexpr std::array<int64_t, N>.
template <auto Arr>
using SeqFromArray = typename detail::SeqFromArrayImpl<Arr>::type;

template <auto... Is>
struct Sequence {
    static constexpr int64_t Size = sizeof...(Is);
    static constexpr std::array<int64_t, sizeof...(Is)> Arr = {static_cast<int64_t>(Is)...};

    static consteval int64_t Product() {
        int64_t p = 1;
        for (auto v : Arr) p *= v;
        return p;
    }
    static consteval int64_t Sum() {
        int64_t s = 0;
        for (auto v : Arr) s += v;
        return s;
    }

    template <auto X>
    using Append = Sequence<Is..., static_cast<int64_t>(X)>;
    template <auto X>
    using Prepend = Sequence<static_cast<int64_t>(X), Is...>;

    template <int I>
    static consteval int64_t Values() {
        static_assert((I < 0 ? Size + I : I) >= 0 && (I < 0 ? Size + I : I) < Size, "Sequence index out of range");
        return Arr[I < 0 ? Size + I : I];
    }
    static consteval int64_t Values(int64_t i) { return Arr[i < 0 ? Size + i : i]; }

    static consteval std::array<int64_t, sizeof...(Is)> Array() { return Arr; }

    static constexpr decltype(auto) Apply(auto&& f) { return f.template operator()<Is...>(); }

    template <typename T>
    consteval operator T() const
        requires(sizeof...(Is) == 1)
    {
        return static_cast<T>(Arr[0]);
    }

  private:
    template <int A, int B>
    static consteval auto swap_arr() {
        auto a = Arr;
        auto t = a[A];
        a[A] = a[B];
        a[B] = t;
        return a;
    }
    template <int N>
    static consteval auto first_arr() {
        std::array<int64_t, N> a{};
        for (int i = 0; i < N; i++) a[i] = Arr[i];
        return a;
    }
    template <int N>
    static consteval auto last_arr() {
        std::array<int64_t, N> a{};
        for (int i = 0; i < N; i++) a[i] = Arr[Size - N + i];
        return a;
    }
    template <int I>
    static consteval auto remove_arr() {
        std::array<int64_t, sizeof...(Is) - 1> a{};
        for (int i = 0, k = 0; i < Size; i++)
            if (i != I) a[k++] = Arr[i];
        return a;
    }
    template <int I, int64_t V>
    static consteval auto insert_arr() {
        std::array<int64_t, sizeof...(Is) + 1> a{};
        for (int i = 0, k = 0; i <= Size; i++) a[i] = (i == I) ? V : Arr[k++];
        return a;
    }
    template <int I, int64_t V>
    static consteval auto set_arr() {
        auto a = Arr;
        a[I] = V;
        return a;
    }

  public:
    template <int A, int B>
    using Swap = SeqFromArray<swap_arr<A, B>()>;
    template <int N>
    using First = SeqFromArray<first_arr<N>()>;
    template <int N>
    using Last = SeqFromArray<last_arr<N>()>;
    template <int I>
    using Remove = SeqFromArray<remove_arr<(I < 0 ? Size + I : I)>()>;
    template <int I, auto V>
    using Insert = SeqFromArray<insert_arr<I, static_cast<int64_t>(V)>()>;
    template <int I, auto V>
    using Set = SeqFromArray<set_arr<(I < 0 ? Size + I : I), static_cast<int64_t>(V)>()>;

    template <auto X>
    static constexpr int IndexOf = [] {
        for (int i = 0; i < Size; i++)
            if (Arr[i] == static_cast<int64_t>(X)) return i;
        return -1;
    }();

    // Every value of Other appears in this sequence, in order (not necessarily adjacent).
    template <typename Other>
    static consteval bool ContainsOrderedSubset() {
        int j = 0;
        for (int i = 0; i < Size && j < Other::Size; i++)
            if (Arr[i] == Other::Arr[j]) j++;
        return j == Other::Size;
    }

    static constexpr bool IsSorted = [] {
        for (int i = 0; i + 1 < Size; i++)
            if (Arr[i] > Arr[i + 1]) return false;
        return true;
    }();

    template <auto... Js>
    consteval bool operator==(Sequence<Js...>) const {
        if constexpr (sizeof...(Js) != sizeof...(Is)) {
            return false;
        } else {
            constexpr std::array<int64_t, sizeof...(Js)> o = {static_cast<int64_t>(Js)...};
            for (int i = 0; i < Size; i++)
                if (Arr[i] != o[i]) return false;
            return true;
        }
    }
};

template <typename A, typename B>
struct ConcatSeq;
template <auto... A, auto... B>
struct ConcatSeq<Sequence<A...>, Sequence<B...>> {
    using type = Sequence<A..., B...>;
};
// Merge: this sequence followed by Seq (reference Sequence.hpp:82-89).
template <typename A, typename B>
using MergeSeq = typename ConcatSeq<A, B>::type;

template <typename T>
concept AnySequence = requires {
    T::Size;
    typename T::template Append<1>;
    typename T::template Prepend<1>;
};

// Row-major strides of Dims (the reference's DefaultStrides, Tensor.hpp:31-40).
template <typename Dims>
consteval auto default_strides_arr() {
    std::array<int64_t, Dims::Size> s{};
    int64_t acc = 1;
    for (int64_t d = Dims::Size - 1; d >= 0; d--) {
        s[d] = acc;
        acc *= Dims::Arr[d];
    }
    return s;
}
template <typename Dims>
using DefaultStrides = SeqFromArray<default_strides_arr<Dims>()>;

static_assert(Sequence<5, 10, 11>::ContainsOrderedSubset<Sequence<5, 11>>(), "ordered-subset sanity");
static_assert(Sequence<2, 3, 4>::Swap<0, 2>() == Sequence<4, 3, 2>());
static_assert(DefaultStrides<Sequence<2, 3, 4>>() == Sequence<12, 4, 1>());

}  // namespace tadma
