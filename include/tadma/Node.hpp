// Node.hpp - user-functor nodes: the reference's Node / make_node /
// MergeNodes / CombineVariadicNode / index_to_value (Node.hpp:14-224,
// Kernels.hpp:10-53, Operations.hpp:299-305), executed by one
// header-templated kernel that the including translation unit compiles for
// sm_100a.  The fixed-function hot path (element-wise chains, reductions,
// norms, gathers) stays in libtadma_b200.so; a node carries an arbitrary C++
// functor, which a C ABI cannot, so its kernel lives here.
//
// A node is (execution shape, functor f, tensors...).  Evaluating it runs
// f(index, tensors...) once per index of the execution shape:
// * an empty shape (Sequence<>) calls f(state, tensors...) once on the host
//   (the reference's input / output marker nodes);
// * a device-capable functor runs in node_kernel on tadma::stream: each
//   thread takes 4 indices 256 apart (coalesced, 4 independent element
//   operations in flight), 64-bit indices, grid-stride beyond 2^31 CTAs;
// * any other functor runs on the host (the reference's CPUExecutor,
//   Node.hpp:14-21): CUDA tensors are staged through host memory.
// A functor is device-capable when it is an nvcc extended lambda (__device__
// or __host__ __device__, --extended-lambda), a class that declares
// `static constexpr bool tadma_device = true`, or an aggregate class (a plain
// functor struct).  nvcc cannot compile an unannotated lambda defined in host
// code for the device ("The closure type for a lambda cannot be used in the
// template argument type of a __global__ function template instantiation"),
// so such a lambda takes the host path.
//
// Tensors reach the kernel as views: a pointer with the static dims and
// strides (DeviceView), or for a trampoline tensor (ExecutionTape::Optimize)
// one value per thread (TrampolineView, the reference's TrampolineStorage,
// Storage.hpp:131-148).  The index a functor receives is a NodeIndex: the
// linear index of the execution shape, whose components idx[d] follow
// MapToShape (Utils.hpp:9-17, last dim fastest).  A view whose layout is
// the execution shape, row-major, addresses element `linear` directly, with
// no per-dimension division.
#pragma once

#include <cuda_runtime.h>

#include <tuple>
#include <type_traits>
#include <utility>
#include <vector>

#include "Tensor.hpp"

// The wrappers below are __host__ __device__ templates around a user functor
// that may be host-only; such a wrapper is then only instantiated for the
// host path, so nvcc's host/device call check is switched off for them.
#ifdef __CUDACC__
#define TADMA_HD_TEMPLATE _Pragma("nv_exec_check_disable")
#else
#define TADMA_HD_TEMPLATE
#endif

namespace tadma {

// ---------------------------------------------------------------- tags --
// A tensor appended to an ExecutionTape carries its tape position in its
// allocator type, so views and copies keep it (Tagging.hpp:7-65).
template <int Tag_, typename Self>
struct Tagged : Self {
    using UntaggedType = Self;
    static constexpr int Tag = Tag_;
};

template <typename T>
concept IsTagged = requires { std::decay_t<T>::Tag; };

template <typename T>
consteval int GetTag() {
    using D = std::decay_t<T>;
    if constexpr (AnyTensor<D>) {
        if constexpr (IsTagged<typename D::Allocator>) return D::Allocator::Tag;
        else return -1;
    } else if constexpr (IsTagged<D>) {
        return D::Tag;
    } else {
        return -1;
    }
}

// A tensor handed out by ExecutionTape::Append: operators on it build nodes
// instead of computing at once (their inputs are produced when the tape runs).
template <typename T>
concept TapeTensor = AnyTensor<T> && (GetTag<T>() >= 0);

template <int Tag, AnyTensor T>
auto AddTag(const T& t) {
    using D = std::decay_t<T>;
    if constexpr (GetTag<D>() == Tag) {
        return t;
    } else {
        static_assert(GetTag<D>() < 0, "Duplicate tag.");
        return Tensor<typename D::ValueType, Tagged<Tag, typename D::Allocator>, typename D::Dims, typename D::Strides>(t.data);
    }
}

template <AnyTensor T>
auto RemoveTag(const T& t) {
    using D = std::decay_t<T>;
    if constexpr (IsTagged<typename D::Allocator>)
        return Tensor<typename D::ValueType, typename D::Allocator::UntaggedType, typename D::Dims, typename D::Strides>(t.data);
    else
        return t;
}

// ------------------------------------------------------------ functors --

template <typename F>
consteval bool device_functor() {
    using D = std::decay_t<F>;
    if constexpr (requires { D::tadma_device; }) {
        return D::tadma_device;
    } else {
#ifdef __CUDACC__
        if constexpr (__nv_is_extended_device_lambda_closure_type(D) || __nv_is_extended_host_device_lambda_closure_type(D))
            return true;
#endif
        return std::is_class_v<D> && std::is_aggregate_v<D>;
    }
}
template <typename F>
constexpr bool device_functor_v = device_functor<F>();

// ------------------------------------------------------------- indices --

template <AnySequence Shape>
struct NodeIndex {
    int64_t linear;
    static constexpr int64_t Size = Shape::Size;

    // Suffix product of the dims after d (the stride of d in row-major order).
    template <int D>
    static consteval int64_t suffix() {
        int64_t p = 1;
        for (int i = D + 1; i < Shape::Size; i++) p *= Shape::Arr[i];
        return p;
    }
    template <int D>
    static consteval int64_t dim() {
        return Shape::Arr[D];
    }
    template <int D>
    __host__ __device__ int64_t component() const {
        if constexpr (Shape::Size == 1) {
            return linear;
        } else {
            constexpr int64_t s = suffix<D>(), n = dim<D>();
            if constexpr (D == 0) return linear / s;
            else return (linear / s) % n;
        }
    }
    template <std::size_t... I>
    __host__ __device__ int64_t pick(int d, std::index_sequence<I...>) const {
        int64_t r = 0;
        ((d == (int)I ? (r = component<(int)I>(), 0) : 0), ...);
        return r;
    }
    // Component d of MapToShape<Shape>(linear) (Utils.hpp:9-17).
    __host__ __device__ int64_t operator[](int d) const { return pick(d, std::make_index_sequence<(std::size_t)Shape::Size>()); }
};

// Same linear index seen through another shape of equal size (ShapeToShape, Utils.hpp:19-27).
template <AnySequence To, AnySequence From>
__host__ __device__ inline NodeIndex<To> reshape_index(const NodeIndex<From>& i) {
    static_assert(To::Product() == From::Product(), "Incompatible shapes");
    return NodeIndex<To>{i.linear};
}

// --------------------------------------------------------------- views --

template <typename T, AnySequence Dims, AnySequence Strides>
struct DeviceView {
    T* p;
    static constexpr int64_t Rank = Dims::Size;
    static constexpr bool Normal = Strides() == DefaultStrides<Dims>();

    template <int D>
    static consteval int64_t stride() { return Strides::Arr[D]; }
    template <std::size_t... I, typename Idx>
    __host__ __device__ int64_t offset(const Idx& idx, std::index_sequence<I...>) const {
        return (int64_t(0) + ... + (idx[(int)I] * stride<(int)I>()));
    }
    // Element at a multi-index of this view's rank (Tensor.hpp:136-154).
    template <AnySequence Shape>
    __host__ __device__ T& operator()(const NodeIndex<Shape>& idx) const {
        static_assert(Shape::Size == Rank, "index rank differs from the tensor's");
        if constexpr (Normal && Shape() == Dims()) return p[idx.linear];
        else return p[offset(idx, std::make_index_sequence<(std::size_t)Rank>())];
    }
    template <typename I, std::size_t N>
    __host__ __device__ T& operator()(const I (&idx)[N]) const {
        static_assert(N == Rank, "index rank differs from the tensor's");
        return p[offset(idx, std::make_index_sequence<N>())];
    }
    template <typename... Is>
        requires(sizeof...(Is) == Rank && (std::is_integral_v<Is> && ...))
    __host__ __device__ T& operator()(Is... is) const {
        const int64_t idx[Rank] = {int64_t(is)...};
        return p[offset(idx, std::make_index_sequence<(std::size_t)Rank>())];
    }
    // Element at a row-major linear index (Tensor.hpp:160-180).
    __host__ __device__ T& operator[](int64_t i) const {
        if constexpr (Normal) {
            return p[i];
        } else {
            return p[linear_offset(i, std::make_index_sequence<(std::size_t)Rank>())];
        }
    }

  private:
    template <std::size_t... I>
    __host__ __device__ static int64_t linear_offset(int64_t i, std::index_sequence<I...>) {
        return (int64_t(0) + ... + (((i / suffix<(int)I>()) % dim<(int)I>()) * stride<(int)I>()));
    }
    template <int D>
    static consteval int64_t dim() {
        return Dims::Arr[D];
    }
    template <int D>
    static consteval int64_t suffix() {
        int64_t s = 1;
        for (int k = D + 1; k < Dims::Size; k++) s *= Dims::Arr[k];
        return s;
    }
};

// A tensor that lives in one register per thread: every index aliases it.
template <typename T>
struct TrampolineView {
    T v;
    template <typename... A>
    __host__ __device__ T& operator()(const A&...) { return v; }
    __host__ __device__ T& operator[](int64_t) { return v; }
};

template <AnyTensor T>
auto make_view(const T& t, typename std::decay_t<T>::ValueType* base = nullptr) {
    using D = std::decay_t<T>;
    using V = typename D::ValueType;
    if constexpr (D::device == kTrampoline) return TrampolineView<V>{};
    else return DeviceView<V, typename D::Dims, typename D::Strides>{base ? base : t.data.view};
}

// Elements a view spans from its base pointer (non-negative strides).
template <AnyTensor T>
consteval int64_t view_extent() {
    using D = std::decay_t<T>;
    if (D::Size == 0) return 0;
    int64_t e = 1;
    for (int i = 0; i < D::Rank; i++) e += (D::Dims::Arr[i] - 1) * D::Strides::Arr[i];
    return e;
}

// --------------------------------------------------------------- kernel --

namespace detail {
constexpr int NODE_THREADS = 256;
constexpr int NODE_PER_THREAD = 4;

// kCUDA if any tensor is on the device, kCPU if any is on the host,
// kTrampoline when every tensor lives in registers, -1 for a mix.
template <typename... Ts>
consteval Memory common_device() {
    const Memory ds[] = {std::decay_t<Ts>::device..., kTrampoline};
    bool cuda = false, cpu = false;
    for (Memory d : ds) {
        cuda = cuda || d == kCUDA;
        cpu = cpu || d == kCPU;
    }
    if (cuda && cpu) return Memory(-1);
    return cuda ? kCUDA : cpu ? kCPU : kTrampoline;
}
}  // namespace detail

#ifdef __CUDACC__
template <AnySequence Shape, typename F, typename... Vs>
__global__ void __launch_bounds__(detail::NODE_THREADS) node_kernel(const F f, const Vs... vs) {
    constexpr int64_t N = Shape::Product();
    constexpr int64_t chunk = (int64_t)detail::NODE_THREADS * detail::NODE_PER_THREAD;
    for (int64_t base = (int64_t)blockIdx.x * chunk + threadIdx.x; base < N; base += (int64_t)gridDim.x * chunk) {
#pragma unroll
        for (int k = 0; k < detail::NODE_PER_THREAD; k++) {
            const int64_t i = base + (int64_t)k * detail::NODE_THREADS;
            if (i < N) {
                // Per-element copies: trampoline values stay in registers.
                [&](Vs... local) { f(NodeIndex<Shape>{i}, local...); }(vs...);
            }
        }
    }
}
#endif

// ----------------------------------------------------------------- Node --

template <typename ExecutionShape_, typename F, typename... Ts>
struct Node {
    std::decay_t<F> f;
    std::tuple<std::decay_t<Ts>...> tensors;
    using ExecutionShape = ExecutionShape_;
    using Functor = std::decay_t<F>;
    static constexpr Memory device = detail::common_device<Ts...>();
    static_assert(device != Memory(-1), "a node mixes CPU and CUDA tensors");

    Node(const F& f_, const Ts&... ts) : f(f_), tensors(ts...) {}

    void Evaluate(auto state) {
        if constexpr (ExecutionShape::Size == 0) {
            std::apply([&](auto&... ts) { f(state, ts...); }, tensors);
        } else if constexpr (device == kTrampoline) {
            // Every tensor lives in registers only: nothing observable to compute.
        } else if constexpr (device == kCUDA && device_functor_v<Functor>) {
#ifdef __CUDACC__
            launch(std::make_index_sequence<sizeof...(Ts)>());
#else
            static_assert(sizeof(F) == 0, "a CUDA node needs nvcc");
#endif
        } else {
            run_on_host(std::make_index_sequence<sizeof...(Ts)>());
        }
    }

    // Tensors this node creates (untagged), or its single tensor
    // (Node.hpp:163-182).
    auto outputs() const {
        if constexpr (sizeof...(Ts) == 1) {
            return tensors;
        } else {
            return outputs_impl<0>(std::tuple<>());
        }
    }
    auto result() const { return std::get<0>(outputs()); }

  private:
    template <std::size_t I, typename Acc>
    auto outputs_impl(Acc acc) const {
        if constexpr (I == sizeof...(Ts)) {
            static_assert(std::tuple_size_v<Acc> > 0, "a node without outputs");
            return acc;
        } else if constexpr (GetTag<std::tuple_element_t<I, std::tuple<std::decay_t<Ts>...>>>() < 0) {
            return outputs_impl<I + 1>(std::tuple_cat(acc, std::tuple{std::get<I>(tensors)}));
        } else {
            return outputs_impl<I + 1>(acc);
        }
    }

#ifdef __CUDACC__
    template <std::size_t... I>
    void launch(std::index_sequence<I...>) {
        constexpr int64_t N = ExecutionShape::Product();
        if constexpr (N > 0) {
            constexpr int64_t per = (int64_t)detail::NODE_THREADS * detail::NODE_PER_THREAD;
            constexpr int64_t want = (N + per - 1) / per;
            constexpr unsigned grid = (unsigned)(want < 0x7fffffff ? want : 0x7fffffff);
            // The functor may read or write any of its tensors.
            (detail::sync_write(std::get<I>(tensors).data.ctl), ...);
            node_kernel<ExecutionShape><<<grid, detail::NODE_THREADS, 0, stream>>>(f, make_view(std::get<I>(tensors))...);
            check_cuda(cudaGetLastError());
        }
    }
#endif

    // The reference's CPUExecutor (Node.hpp:14-21).  CUDA tensors are copied to
    // host buffers first and back afterwards.
    template <std::size_t... I>
    void run_on_host(std::index_sequence<I...>) {
        constexpr int64_t N = ExecutionShape::Product();
        (detail::sync_write(std::get<I>(tensors).data.ctl), ...);
        if constexpr (device == kCUDA) {
            auto host = std::make_tuple(stage_in<I>()...);
            check_cuda(cudaStreamSynchronize(stream));
            for (int64_t i = 0; i < N; i++) {
                auto vs = std::make_tuple(make_view(std::get<I>(tensors), host_ptr<I>(std::get<I>(host)))...);
                f(NodeIndex<ExecutionShape>{i}, std::get<I>(vs)...);
            }
            (stage_out<I>(std::get<I>(host)), ...);
        } else {
            for (int64_t i = 0; i < N; i++) {
                auto vs = std::make_tuple(make_view(std::get<I>(tensors))...);
                f(NodeIndex<ExecutionShape>{i}, std::get<I>(vs)...);
            }
        }
    }
    template <std::size_t I>
    auto stage_in() {
        using TT = std::tuple_element_t<I, std::tuple<std::decay_t<Ts>...>>;
        using V = typename TT::ValueType;
        std::vector<V> buf;
        if constexpr (TT::device == kCUDA) {
            constexpr int64_t n = view_extent<TT>();
            buf.resize((std::size_t)n);
            if (n > 0)
                check_cuda(cudaMemcpyAsync(buf.data(), std::get<I>(tensors).data.view, sizeof(V) * n, cudaMemcpyDeviceToHost, stream));
        }
        return buf;
    }
    template <std::size_t I, typename V>
    V* host_ptr(std::vector<V>& buf) {
        return buf.empty() ? nullptr : buf.data();
    }
    template <std::size_t I, typename V>
    void stage_out(const std::vector<V>& buf) {
        using TT = std::tuple_element_t<I, std::tuple<std::decay_t<Ts>...>>;
        if constexpr (TT::device == kCUDA) {
            if (!buf.empty())
                check_cuda(cudaMemcpyAsync(std::get<I>(tensors).data.view, buf.data(), sizeof(V) * buf.size(),
                                           cudaMemcpyHostToDevice, stream));
            check_cuda(cudaStreamSynchronize(stream));
        }
    }
};

template <AnySequence ExecutionShape>
auto make_node(auto&& f, auto&&... tensors) {
    return Node<ExecutionShape, std::decay_t<decltype(f)>, std::decay_t<decltype(tensors)>...>(f, tensors...);
}

template <typename T>
concept IsNode = requires { typename std::decay_t<T>::ExecutionShape; };

// ------------------------------------------------------------ MergeNodes --
// Two nodes of equal execution size become one kernel: each index runs the
// first functor, then the second (Node.hpp:189-224).  Tensors with the same
// tag and type appear once in the merged node.

namespace detail {

template <std::size_t I, typename A, typename... R>
__host__ __device__ auto& nth(A& a, R&... r) {
    if constexpr (I == 0) return a;
    else return nth<I - 1>(r...);
}

template <typename Tuple, std::size_t... K>
consteval auto same_type_table(std::index_sequence<K...>) {
    constexpr std::size_t n = std::tuple_size_v<Tuple>;
    std::array<bool, n * n> s{};
    ((s[K] = std::is_same_v<std::tuple_element_t<K / n, Tuple>, std::tuple_element_t<K % n, Tuple>>), ...);
    return s;
}
template <typename Tuple, std::size_t... I>
consteval auto tag_table(std::index_sequence<I...>) {
    std::array<int, sizeof...(I)> t{};
    ((t[I] = GetTag<std::tuple_element_t<I, Tuple>>()), ...);
    return t;
}

// Position of each tensor of the concatenated tuple in the merged tuple: a
// tagged tensor seen before (same tag, same type) reuses that position.
template <typename Tuple>
consteval auto merge_mapping() {
    constexpr std::size_t n = std::tuple_size_v<Tuple>;
    const auto tags = tag_table<Tuple>(std::make_index_sequence<n>());
    const auto same = same_type_table<Tuple>(std::make_index_sequence<n * n>());
    std::array<int, n> out{};
    int next = 0;
    for (std::size_t i = 0; i < n; i++) {
        out[i] = -1;
        if (tags[i] >= 0)
            for (std::size_t j = 0; j < i && out[i] < 0; j++)
                if (tags[j] == tags[i] && same[i * n + j]) out[i] = out[j];
        if (out[i] < 0) out[i] = next++;
    }
    return out;
}

template <typename Tuple, std::size_t Off, std::size_t... I>
auto merge_positions(std::index_sequence<I...>) -> std::index_sequence<(std::size_t)merge_mapping<Tuple>()[Off + I]...>;

template <typename Tuple>
consteval auto merge_keep() {
    constexpr auto m = merge_mapping<Tuple>();
    std::array<bool, m.size()> keep{};
    int seen = 0;
    for (std::size_t i = 0; i < m.size(); i++) {
        keep[i] = m[i] == seen;
        if (keep[i]) seen++;
    }
    return keep;
}

template <typename Tuple, std::size_t I = 0>
auto fold_tuple(const Tuple& t) {
    constexpr auto keep = merge_keep<Tuple>();
    if constexpr (I == std::tuple_size_v<Tuple>) {
        return std::tuple<>();
    } else if constexpr (keep[I]) {
        return std::tuple_cat(std::tuple{std::get<I>(t)}, fold_tuple<Tuple, I + 1>(t));
    } else {
        return fold_tuple<Tuple, I + 1>(t);
    }
}

// f0 over the first node's tensors, then f1 over the second's; M0 / M1 give
// each node's tensors' positions in the merged tuple.
template <typename S0, typename S1, typename F0, typename F1, typename M0, typename M1>
struct Merged;
template <typename S0, typename S1, typename F0, typename F1, std::size_t... A, std::size_t... B>
struct Merged<S0, S1, F0, F1, std::index_sequence<A...>, std::index_sequence<B...>> {
    F0 f0;
    F1 f1;
    static constexpr bool tadma_device = device_functor_v<F0> && device_functor_v<F1>;
    Merged(const F0& a, const F1& b) : f0(a), f1(b) {}

    TADMA_HD_TEMPLATE
    template <typename Idx, typename... Vs>
    __host__ __device__ void operator()(const Idx& idx, Vs&... vs) const {
        f0(idx, nth<A>(vs...)...);
        if constexpr (std::is_same_v<S0, S1>) f1(idx, nth<B>(vs...)...);
        else f1(reshape_index<S1>(idx), nth<B>(vs...)...);
    }
};

}  // namespace detail

template <typename N0, typename N1>
auto MergeNodes(const N0& n0, const N1& n1) {
    using S0 = typename N0::ExecutionShape;
    using S1 = typename N1::ExecutionShape;
    static_assert(S0::Product() == S1::Product(), "Incompatible shapes");
    auto trivial = std::tuple_cat(n0.tensors, n1.tensors);
    using TT = decltype(trivial);
    constexpr std::size_t n0s = std::tuple_size_v<decltype(n0.tensors)>;
    constexpr std::size_t n1s = std::tuple_size_v<decltype(n1.tensors)>;
    using M0 = decltype(detail::merge_positions<TT, 0>(std::make_index_sequence<n0s>()));
    using M1 = decltype(detail::merge_positions<TT, n0s>(std::make_index_sequence<n1s>()));
    using F = detail::Merged<S0, S1, typename N0::Functor, typename N1::Functor, M0, M1>;
    auto folded = detail::fold_tuple(trivial);
    return std::apply([&](const auto&... ts) { return make_node<S0>(F(n0.f, n1.f), ts...); }, folded);
}

template <typename N0, typename N1, typename... Ns>
    requires(sizeof...(Ns) > 0)
auto MergeNodes(const N0& n0, const N1& n1, const Ns&... ns) {
    return MergeNodes(MergeNodes(n0, n1), ns...);
}

// ----------------------------------------------- node builders (Kernels.hpp) --

namespace nodefn {

// f(tensors(index)...) for every index (the lambda of CombineVariadicNode,
// Kernels.hpp:10-14).
template <typename F>
struct ApplyAt {
    F f;
    static constexpr bool tadma_device = device_functor_v<F>;
    explicit ApplyAt(const F& f_) : f(f_) {}
    TADMA_HD_TEMPLATE
    template <typename Idx, typename... Vs>
    __host__ __device__ void operator()(const Idx& idx, Vs&... vs) const {
        f(vs(idx)...);
    }
};

// x = f(x) (InplaceNode), y = f(x) (EltwiseNode), x = f(x, y) (CombineNode),
// z = f(x, y) (CombineToNode).
template <typename F>
struct SetUnary {
    F f;
    static constexpr bool tadma_device = device_functor_v<F>;
    explicit SetUnary(const F& f_) : f(f_) {}
    TADMA_HD_TEMPLATE
    template <typename X>
    __host__ __device__ void operator()(X& x) const { x = f(x); }
};
template <typename F>
struct MapUnary {
    F f;
    static constexpr bool tadma_device = device_functor_v<F>;
    explicit MapUnary(const F& f_) : f(f_) {}
    TADMA_HD_TEMPLATE
    template <typename X, typename Y>
    __host__ __device__ void operator()(const X& x, Y& y) const { y = f(x); }
};
template <typename F>
struct SetBinary {
    F f;
    static constexpr bool tadma_device = device_functor_v<F>;
    explicit SetBinary(const F& f_) : f(f_) {}
    TADMA_HD_TEMPLATE
    template <typename X, typename Y>
    __host__ __device__ void operator()(X& x, const Y& y) const { x = f(x, y); }
};
template <typename F>
struct MapBinary {
    F f;
    static constexpr bool tadma_device = device_functor_v<F>;
    explicit MapBinary(const F& f_) : f(f_) {}
    TADMA_HD_TEMPLATE
    template <typename X, typename Y, typename Z>
    __host__ __device__ void operator()(const X& x, const Y& y, Z& z) const { z = f(x, y); }
};

// result[index] = f(index) over a flat execution shape (Operations.hpp:299-305).
template <typename F>
struct IndexToValue {
    F f;
    static constexpr bool tadma_device = device_functor_v<F>;
    explicit IndexToValue(const F& f_) : f(f_) {}
    TADMA_HD_TEMPLATE
    template <typename Idx, typename R>
    __host__ __device__ void operator()(const Idx& idx, R& result) const { result[idx[0]] = f(idx[0]); }
};

}  // namespace nodefn

// A node of t0's shape calling f(t0(i), ts(i)...) with the others broadcast
// to t0 (Kernels.hpp:10-14).
template <AnyTensor T0, AnyTensor... Ts>
auto CombineVariadicNode(const auto& f, const T0& t0, const Ts&... ts) {
    using F = std::decay_t<decltype(f)>;
    return make_node<typename T0::Dims>(nodefn::ApplyAt<F>(f), t0, ts.template broadcastTo<typename T0::Dims>()...);
}

template <AnyTensor T>
auto InplaceNode(const T& t, const auto& f) {
    using F = std::decay_t<decltype(f)>;
    return CombineVariadicNode(nodefn::SetUnary<F>(f), t.removeFakeDims());
}

template <AnyTensor T>
auto EltwiseNode(const T& x, const auto& f) {
    using F = std::decay_t<decltype(f)>;
    using R = std::decay_t<decltype(f(typename T::ValueType()))>;
    using A = std::conditional_t<IsTagged<typename T::Allocator>, typename T::Allocator::UntaggedType, typename T::Allocator>;
    Tensor<R, A, typename T::Dims> y;
    return CombineVariadicNode(nodefn::MapUnary<F>(f), x, y);
}

template <AnyTensor T1, AnyTensor T2>
auto CombineNode(const T1& x, const T2& y, const auto& f) {
    using F = std::decay_t<decltype(f)>;
    return CombineVariadicNode(nodefn::SetBinary<F>(f), x, y);
}

template <typename F>
concept CommutativeFn = requires { std::decay_t<F>::commutative; } && std::decay_t<F>::commutative;

template <AnyTensor T1, AnyTensor T2>
auto CombineToNode(const T1& x, const T2& y, const auto& f) {
    using F = std::decay_t<decltype(f)>;
    using R = std::decay_t<decltype(f(typename T1::ValueType(), typename T2::ValueType()))>;
    if constexpr (!Broadcastable<T2, T1> && Broadcastable<T1, T2> && CommutativeFn<F>) {
        return CombineToNode(y, x, f);
    } else {
        using A = std::conditional_t<IsTagged<typename T1::Allocator>, typename T1::Allocator::UntaggedType,
                                     typename T1::Allocator>;
        Tensor<R, A, typename T1::Dims> z;
        return CombineVariadicNode(nodefn::MapBinary<F>(f), x, y.template broadcastTo<typename T1::Dims>(), z);
    }
}

template <bool Inplace, AnyTensor T>
auto MakeEltwiseNode(const T& x, const auto& f) {
    if constexpr (Inplace) return InplaceNode(x, f);
    else return EltwiseNode(x, f);
}

// A node writing f(i) to element i of a new tensor of Shape on `device`.
template <AnySequence Shape, Memory device>
auto index_to_value(auto&& f) {
    using F = std::decay_t<decltype(f)>;
    using R = std::decay_t<decltype(f(0))>;
    Tensor<R, Allocator<device>, Shape> result;
    return make_node<Sequence<Shape::Product()>>(nodefn::IndexToValue<F>(f), result);
}

}  // namespace tadma
