// ExecutionTape.hpp - a compile-time linearised graph of nodes (the
// reference's ExecutionTape, ExecutionTape.hpp:26-192).
//
//   auto [tape2, t1] = tape.Append(node);   // t1: node's new tensors, tagged
//   auto graph = tapeN.Optimize();           // single-use tensors -> registers
//   graph.Evaluate(state);                   // every node, in order
//   graph.Last();                            // the last node
//
// Append tags every tensor the node creates with its tape position (in the
// tensor's allocator type), then merges the node into an earlier one when
// that is safe, so both run as one kernel (MergeNodes).  Merge rule:
// * both nodes run on the device (device-capable functors, CUDA tensors) and
//   have execution shapes of equal size;
// * the target node is the latest node that shares a tensor with the new one,
//   or comes after it (so every producer of the new node's inputs runs no
//   later than the merged kernel), the one sharing the most tensors, the
//   later one on ties (FindMergeable, ExecutionTape.hpp:131-192);
// * every shared tensor is row-major and has exactly one element per index
//   of the execution shape, so each thread reads only what it wrote itself.
//   The reference merges on equal size alone and documents the race this
//   leaves (ExecutionTape.hpp:178-181); this build does not merge there.
// Optimize replaces each tensor referenced by one node only with a
// trampoline: a register per thread, no memory (ExecutionTape.hpp:74-102).  A
// tensor the tape reads but did not create must be registered by a node of
// its own (an input node, as the reference's demo does), or it is treated as
// a single-use intermediate.
#pragma once

#include <algorithm>
#include <tuple>

#include "Node.hpp"

namespace tadma {

namespace detail {

template <typename Tuple, int Start, std::size_t... I>
consteval auto assign_tags(std::index_sequence<I...>) {
    std::array<int, sizeof...(I)> tags{};
    ((tags[I] = GetTag<std::tuple_element_t<I, Tuple>>()), ...);
    int next = Start;
    for (auto& t : tags)
        if (t < 0) t = next++;
    return tags;
}

template <typename Tuple, int Start>
constexpr auto assigned_tags = assign_tags<Tuple, Start>(std::make_index_sequence<std::tuple_size_v<Tuple>>());

template <typename N>
consteval bool runs_on_device() {
    return N::ExecutionShape::Size > 0 && N::device == kCUDA && device_functor_v<typename N::Functor>;
}

// Number of tensors of node N (by tag) that node M also holds.
template <typename N, typename M>
consteval int shared_tensors() {
    using TN = decltype(std::declval<N>().tensors);
    using TM = decltype(std::declval<M>().tensors);
    const auto tn = tag_table<TN>(std::make_index_sequence<std::tuple_size_v<TN>>());
    const auto tm = tag_table<TM>(std::make_index_sequence<std::tuple_size_v<TM>>());
    int c = 0;
    for (int a : tn)
        for (int b : tm)
            if (a >= 0 && a == b) {
                c++;
                break;
            }
    return c;
}

// Every tensor N and M share is row-major with one element per index.
template <typename N, typename M, std::size_t... I>
consteval bool shared_are_elementwise(std::index_sequence<I...>) {
    using TN = decltype(std::declval<N>().tensors);
    using TM = decltype(std::declval<M>().tensors);
    const auto tm = tag_table<TM>(std::make_index_sequence<std::tuple_size_v<TM>>());
    constexpr int64_t P = N::ExecutionShape::Product();
    auto ok_one = [&](int tag, bool normal, int64_t size) {
        if (tag < 0) return true;
        for (int b : tm)
            if (b == tag) return normal && size == P;
        return true;
    };
    return (ok_one(GetTag<std::tuple_element_t<I, TN>>(), std::tuple_element_t<I, TN>::NormalStrides,
                   std::tuple_element_t<I, TN>::Size) &&
            ...);
}
template <typename N, typename M>
consteval bool shared_are_elementwise() {
    using TN = decltype(std::declval<N>().tensors);
    using TM = decltype(std::declval<M>().tensors);
    return shared_are_elementwise<N, M>(std::make_index_sequence<std::tuple_size_v<TN>>()) &&
           shared_are_elementwise<M, N>(std::make_index_sequence<std::tuple_size_v<TM>>());
}

template <typename Tuple, std::size_t J, typename T>
consteval bool tuple_has_tag(int tag) {
    using TT = decltype(std::declval<std::tuple_element_t<J, Tuple>>().tensors);
    const auto tags = tag_table<TT>(std::make_index_sequence<std::tuple_size_v<TT>>());
    for (int t : tags)
        if (t == tag) return true;
    return false;
}

}  // namespace detail

template <int NextTag = 0, typename TupleType_ = std::tuple<>>
struct ExecutionTape {
    using TupleType = TupleType_;
    TupleType data;
    static constexpr auto Size = std::tuple_size_v<TupleType>;

    ExecutionTape() = default;
    explicit ExecutionTape(const TupleType& tuple) : data(tuple) {}

    // Append a node: returns {new tape, the node's new tensors (tagged)...}.
    template <bool DoNotMerge = false, typename N>
    auto Append(const N& node0) {
        using NodeT = std::decay_t<N>;
        using NodeTuple = decltype(node0.tensors);
        constexpr auto tags = detail::assigned_tags<NodeTuple, NextTag + 1>;
        auto tagged = tag_all(node0.tensors, std::make_index_sequence<std::tuple_size_v<NodeTuple>>());
        auto full = std::apply(
            [&](const auto&... ts) { return make_node<typename NodeT::ExecutionShape>(node0.f, ts...); }, tagged);
        using Full = decltype(full);
        constexpr int merge_index = DoNotMerge ? -1 : FindMergeable<Full>();
        constexpr int next_next = std::max(NextTag + 1, max_of(tags) + 1);
        auto outs = outputs_of<NodeTuple>(tagged, std::make_index_sequence<std::tuple_size_v<NodeTuple>>());
        if constexpr (merge_index < 0) {
            auto nd = std::tuple_cat(data, std::tuple{full});
            return std::tuple_cat(std::tuple{ExecutionTape<next_next, decltype(nd)>(nd)}, outs);
        } else {
            auto nd = replace<merge_index>(data, MergeNodes(std::get<merge_index>(data), full),
                                           std::make_index_sequence<Size>());
            return std::tuple_cat(std::tuple{ExecutionTape<next_next, decltype(nd)>(nd)}, outs);
        }
    }

    // Tensors referenced by one node only become trampolines.
    auto Optimize() const {
        auto nd = optimize_nodes(std::make_index_sequence<Size>());
        return ExecutionTape<NextTag, decltype(nd)>(nd);
    }

    void Evaluate(auto state) {
        std::apply([&](auto&... nodes) { (nodes.Evaluate(state), ...); }, data);
    }

    auto& Last() { return std::get<Size - 1>(data); }

  private:
    static consteval int max_of(const auto& a) {
        int m = -1;
        for (int v : a) m = v > m ? v : m;
        return m;
    }

    template <typename Tuple, std::size_t... I>
    static auto tag_all(const Tuple& t, std::index_sequence<I...>) {
        constexpr auto tags = detail::assigned_tags<Tuple, NextTag + 1>;
        return std::make_tuple(AddTag<tags[I]>(std::get<I>(t))...);
    }

    // The node's outputs: the tensors it created (untagged before Append), or
    // its single tensor (Node.hpp:163-182).
    template <typename Orig, typename Tagged, std::size_t... I>
    static auto outputs_of(const Tagged& tagged, std::index_sequence<I...>) {
        if constexpr (sizeof...(I) == 1) {
            return tagged;
        } else {
            return std::tuple_cat([&] {
                if constexpr (GetTag<std::tuple_element_t<I, Orig>>() < 0) return std::tuple{std::get<I>(tagged)};
                else return std::tuple<>();
            }()...);
        }
    }

    template <std::size_t K, typename Tuple, typename V, std::size_t... I>
    static auto replace(const Tuple& t, const V& v, std::index_sequence<I...>) {
        return std::make_tuple([&]() -> decltype(auto) {
            if constexpr (I == K) return v;
            else return std::get<I>(t);
        }()...);
    }

    template <typename Node>
    static consteval int FindMergeable() {
        if constexpr (!detail::runs_on_device<Node>()) {
            return -1;
        } else {
            return find_mergeable<Node>(std::make_index_sequence<Size>());
        }
    }
    template <typename Node, std::size_t... I>
    static consteval int find_mergeable(std::index_sequence<I...>) {
        constexpr int n = (int)Size;
        int shares[n > 0 ? n : 1] = {detail::shared_tensors<Node, std::tuple_element_t<I, TupleType>>()...};
        bool ok[n > 0 ? n : 1] = {(detail::runs_on_device<std::tuple_element_t<I, TupleType>>() &&
                                   std::tuple_element_t<I, TupleType>::ExecutionShape::Product() ==
                                       Node::ExecutionShape::Product() &&
                                   detail::shared_are_elementwise<Node, std::tuple_element_t<I, TupleType>>())...};
        int latest_share = -1;
        for (int i = 0; i < n; i++)
            if (shares[i] > 0) latest_share = i;
        int best = -1, best_score = -1;
        for (int i = n - 1; i >= 0 && i >= latest_share; i--) {
            if (ok[i] && shares[i] > best_score) {
                best = i;
                best_score = shares[i];
            }
        }
        return best;
    }

    static consteval auto tensor_refs() {
        std::array<int, NextTag + 1> refs{};
        count_refs(refs, std::make_index_sequence<Size>());
        return refs;
    }
    template <std::size_t... I>
    static consteval void count_refs(std::array<int, NextTag + 1>& refs, std::index_sequence<I...>) {
        (count_node<std::tuple_element_t<I, TupleType>>(refs), ...);
    }
    template <typename N>
    static consteval void count_node(std::array<int, NextTag + 1>& refs) {
        using TT = decltype(std::declval<N>().tensors);
        const auto tags = tag_table<TT>(std::make_index_sequence<std::tuple_size_v<TT>>());
        for (int t : tags)
            if (t >= 0 && t <= NextTag) refs[t]++;
    }
    template <typename Tuple>
    static consteval auto tag_table(auto seq) {
        return detail::tag_table<Tuple>(seq);
    }

    template <std::size_t... I>
    auto optimize_nodes(std::index_sequence<I...>) const {
        return std::make_tuple(optimize_node(std::get<I>(data))...);
    }
    template <typename N>
    static auto optimize_node(const N& node) {
        constexpr auto refs = tensor_refs();
        return std::apply(
            [&](const auto&... ts) {
                return make_node<typename N::ExecutionShape>(node.f, trampoline_if_single<refs>(ts)...);
            },
            node.tensors);
    }
    template <auto Refs, typename T>
    static auto trampoline_if_single(const T& t) {
        constexpr int tag = GetTag<T>();
        if constexpr (tag >= 0 && Refs[tag] == 1) {
            return Tensor<typename T::ValueType, Allocator<kTrampoline>, typename T::Dims>();
        } else {
            return t;
        }
    }
};

}  // namespace tadma
