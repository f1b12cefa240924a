// Tensor.hpp - the static-shape Tensor: dims and strides are types, views are
// free, every computing op lowers to one call of libtadma_b200.so.
//
// Mirrors the reference's Tensor (include/tadma/Tensor.hpp:20-453) and keeps
// its spellings: Tensor<T, Allocator<kCUDA>, Sequence<dims...>[, Sequence<strides...>]>,
// Dims / Strides / Rank / Size / NormalStrides / HasBroadcastDims, Dim(i),
// Stride(i), transpose, slice, squeeze, unsqueeze, broadcast, broadcastTo,
// reshape, index, split, clone, contiguous, to<Memory>, to<U>, copyTo,
// sum / min / max / mean, operator<<, CpuTensor / CudaTensor.  Differences
// (each deliberate, see the comments at each member):
// * C++20 instead of C++23 (nvcc 12.9): members take `const&` this instead of
//   deducing-this;
// * transpose<P...>() with Rank arguments is a permutation (generated code
//   emits transpose<0,2,1,3>, which the reference lacks); with exactly two
//   arguments it swaps two axes, as the reference's transpose<D0,D1>;
// * squeeze<Dims...>() works (the reference's body is empty);
// * argmax / argmin reductions are new;
// * mean<-1> normalises the axis (the reference calls Dim(D) with D < 0).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <array>
#include <cstring>
#include <fstream>
#include <iostream>
#include <tuple>
#include <type_traits>
#include <vector>

#include "Core.hpp"
#include "Deferred.hpp"
#include "Sequence.hpp"

namespace tadma {

// ------------------------------------------------------------- dtypes --

template <typename T>
struct DTypeOf {};
template <> struct DTypeOf<float> { static constexpr int value = TADMA_F32; };
template <> struct DTypeOf<__half> { static constexpr int value = TADMA_F16; };
template <> struct DTypeOf<__nv_bfloat16> { static constexpr int value = TADMA_BF16; };
template <> struct DTypeOf<double> { static constexpr int value = TADMA_F64; };
template <> struct DTypeOf<int64_t> { static constexpr int value = TADMA_I64; };
template <> struct DTypeOf<int32_t> { static constexpr int value = TADMA_I32; };
template <> struct DTypeOf<uint8_t> { static constexpr int value = TADMA_U8; };
template <> struct DTypeOf<bool> { static constexpr int value = TADMA_BOOL; };
template <> struct DTypeOf<int8_t> { static constexpr int value = TADMA_I8; };

template <typename T>
concept Element = requires { DTypeOf<T>::value; };
template <typename T>
constexpr int dtype_v = DTypeOf<T>::value;

// A scalar operand: an arithmetic value, or a compile-time value holder of the
// generated code (ConstexprHolder<v>: `x + _LayerNorm_Constant_1_output_0`).
template <typename T>
concept HeldScalar = requires {
    typename T::ValueType;
    T::value;
} && std::is_arithmetic_v<typename T::ValueType>;
template <typename T>
concept Scalar = std::is_arithmetic_v<T> || HeldScalar<T>;

namespace detail {
template <typename S>
struct scalar_type {
    using type = S;
};
template <HeldScalar S>
struct scalar_type<S> {
    using type = typename S::ValueType;
};
}  // namespace detail
// The arithmetic type of a scalar operand.
template <typename S>
using scalar_t = typename detail::scalar_type<S>::type;

// ------------------------------------------------------- layout algebra --

template <typename Dims, typename Strides>
consteval bool has_broadcast_dims() {
    for (int i = 0; i < Dims::Size; i++)
        if (Strides::Arr[i] == 0 && Dims::Arr[i] != 1) return true;
    return false;
}

// Result of removeFakeDims (Tensor.hpp:242-249): drop dims of extent 1 or stride 0.
template <typename Dims, typename Strides>
consteval int fake_free_rank() {
    int r = 0;
    for (int i = 0; i < Dims::Size; i++)
        if (Dims::Arr[i] != 1 && Strides::Arr[i] != 0) r++;
    return r;
}
template <typename Dims, typename Strides, bool WantStrides>
consteval auto fake_free_arr() {
    std::array<int64_t, fake_free_rank<Dims, Strides>()> a{};
    for (int i = 0, k = 0; i < Dims::Size; i++)
        if (Dims::Arr[i] != 1 && Strides::Arr[i] != 0) a[k++] = WantStrides ? Strides::Arr[i] : Dims::Arr[i];
    return a;
}

// broadcastTo (Tensor.hpp:383-406): the non-fake dims of the source must
// appear in order in the target; every other target dim gets stride 0.
template <typename Dims, typename Strides, typename Target>
consteval bool broadcastable_to() {
    if (Dims() == Target()) return true;
    if (Dims::Size == 1 && Dims::Arr[0] == 1) return true;
    using CD = SeqFromArray<fake_free_arr<Dims, Strides, false>()>;
    return Target::template ContainsOrderedSubset<CD>();
}
template <typename Dims, typename Strides, typename Target>
consteval auto broadcast_strides_arr() {
    std::array<int64_t, Target::Size> out{};
    if constexpr (Dims() == Target()) {
        for (int i = 0; i < Target::Size; i++) out[i] = Strides::Arr[i];
    } else {
        constexpr auto cd = fake_free_arr<Dims, Strides, false>();
        constexpr auto cs = fake_free_arr<Dims, Strides, true>();
        int j = 0;
        for (int i = 0; i < Target::Size; i++) {
            if (j < (int)cd.size() && cd[j] == Target::Arr[i]) out[i] = cs[j++];
            else out[i] = 0;
        }
    }
    return out;
}

// Values of one reshape<...> argument: an integer, or a compile-time shape
// value whose type carries them (Vals::Arr of a ConstTensor, value of a holder).
template <auto X>
consteval auto shape_arg_values() {
    using XT = std::remove_cvref_t<decltype(X)>;  // a class-type template argument is const
    if constexpr (requires { XT::Vals::Arr; }) return XT::Vals::Arr;
    else if constexpr (requires { XT::value; }) return std::array<int64_t, 1>{static_cast<int64_t>(XT::value)};
    else return std::array<int64_t, 1>{static_cast<int64_t>(X)};
}
template <auto X>
consteval std::size_t shape_arg_size() {
    return shape_arg_values<X>().size();
}

template <typename Dims, int... P>
consteval auto permute_arr(const std::array<int64_t, Dims::Size>& src) {
    std::array<int64_t, Dims::Size> out{};
    constexpr int p[] = {P...};
    for (int i = 0; i < Dims::Size; i++) out[i] = src[p[i] < 0 ? p[i] + Dims::Size : p[i]];
    return out;
}

template <typename Dims>
consteval auto reversed_arr(const std::array<int64_t, Dims::Size>& src) {
    std::array<int64_t, Dims::Size> out{};
    for (int i = 0; i < Dims::Size; i++) out[i] = src[Dims::Size - 1 - i];
    return out;
}

// ------------------------------------------------------ weight staging --

namespace detail {

// Pinned host slots through which weight files reach the device: slot k is
// refilled only after its previous copy has completed (its event), so file
// reads overlap the host-to-device copies of earlier slots.  One per thread,
// created on the first CUDA weight load; released at thread exit.
struct WeightStager {
    static constexpr int kSlots = 4;
    static constexpr int64_t kSlotBytes = 16 << 20;
    char* slot[kSlots] = {};
    cudaEvent_t done[kSlots] = {};
    bool pending[kSlots] = {};
    int next = 0;

    void load(std::ifstream& file, char* dst, int64_t bytes, cudaStream_t s) {
        if (!slot[0]) {
            for (int k = 0; k < kSlots; k++) {
                check_cuda(cudaMallocHost(reinterpret_cast<void**>(&slot[k]), kSlotBytes));
                check_cuda(cudaEventCreateWithFlags(&done[k], cudaEventDisableTiming));
            }
        }
        for (int64_t off = 0; off < bytes; off += kSlotBytes) {
            const int64_t n = bytes - off < kSlotBytes ? bytes - off : kSlotBytes;
            const int k = next;
            next = (next + 1) % kSlots;
            if (pending[k]) check_cuda(cudaEventSynchronize(done[k]));
            pending[k] = false;
            file.read(slot[k], n);
            if (!file) throw std::runtime_error("tadma: weight file read failed");
            check_cuda(cudaMemcpyAsync(dst + off, slot[k], (size_t)n, cudaMemcpyHostToDevice, s));
            check_cuda(cudaEventRecord(done[k], s));
            pending[k] = true;
        }
    }
    ~WeightStager() {
        for (int k = 0; k < kSlots; k++) {
            if (pending[k]) cudaEventSynchronize(done[k]);
            if (done[k]) cudaEventDestroy(done[k]);
            if (slot[k]) cudaFreeHost(slot[k]);
        }
    }
};

inline WeightStager& weight_stager() {
    static thread_local WeightStager stager;
    return stager;
}

}  // namespace detail

// -------------------------------------------------------------- Tensor --

template <typename T, typename Allocator_, AnySequence Dims_, AnySequence StridesInit = Sequence<>>
struct Tensor;

template <typename T>
concept AnyTensor = requires {
    std::decay_t<T>::Rank;
    typename std::decay_t<T>::Dims;
    typename std::decay_t<T>::Strides;
    std::decay_t<T>::device;
};

template <typename T>
concept AnyCudaTensor = AnyTensor<T> && (std::decay_t<T>::device == kCUDA);

template <typename T, typename Allocator_, AnySequence Dims_, AnySequence StridesInit>
struct Tensor {
    using Allocator = Allocator_;
    using AllocatorType = Allocator_;
    static constexpr Memory device = Allocator::device;
    using ValueType = T;
    using Dims = Dims_;
    static constexpr int64_t Rank = Dims::Size;
    static constexpr int64_t Size = Dims::Product();
    static constexpr int64_t SizeBytes = int64_t(sizeof(T)) * Size;
    using Strides = std::conditional_t<(StridesInit::Size == 0 && Rank > 0), DefaultStrides<Dims>, StridesInit>;
    static constexpr bool NormalStrides = (Strides() == DefaultStrides<Dims>());
    static constexpr bool HasBroadcastDims = has_broadcast_dims<Dims, Strides>();
    static constexpr bool IsScalar = Size == 1;
    static_assert(Rank <= TADMA_MAX_RANK, "rank above 8 is not supported");
    static_assert(Element<T>, "element type must be one of float, __half, __nv_bfloat16, double, int64_t, int32_t, "
                              "uint8_t, bool, int8_t");

    HeapStorage<T> data;

    static consteval int64_t Dim(int i) { return Dims::Values(i < 0 ? i + Rank : i); }
    static consteval int64_t Stride(int i) { return Strides::Values(i < 0 ? i + Rank : i); }

    // ----------------------------------------------------- construction --
    // Allocates Size elements with the tensor's allocator (a new, owning tensor).
    Tensor() : data(Allocator::template allocate<T, Size>()) {}
    explicit Tensor(const HeapStorage<T>& s) : data(s) {}
    // Non-owning wrap of an existing buffer (Tensor.hpp:74-78).
    Tensor(const T* p) : data(const_cast<T*>(p)) {}
    Tensor(void* p) : data(static_cast<T*>(p)) {}
    Tensor(const Tensor&) = default;
    Tensor(Tensor&&) noexcept = default;
    Tensor& operator=(Tensor&& o) noexcept {
        std::swap(data, o.data);
        return *this;
    }
    Tensor& operator=(const Tensor& o) = default;

    // Weight load: SizeBytes at `offset` of a flat little-endian file, the
    // layout the ONNX-to-C++ generator writes (raw tensors back to back,
    // cppgen.py:111-116; the reference's loader, Tensor.hpp:86-99, allocates,
    // copies and synchronises once per tensor).  A CUDA tensor streams through
    // the calling thread's ring of pinned staging slots (detail::WeightStager):
    // the file is read into one slot while earlier slots copy to the device,
    // and nothing synchronises per tensor; ops on tadma::stream are ordered
    // after the copies.
    Tensor(std::ifstream& file, uint64_t offset) : Tensor() {
        static_assert(NormalStrides, "weights load into a contiguous tensor");
        file.seekg((std::streamoff)offset);
        if constexpr (device == kCPU) {
            file.read(reinterpret_cast<char*>(data.view), SizeBytes);
            if (!file) throw std::runtime_error("tadma: weight file read failed");
        } else {
            detail::weight_stager().load(file, reinterpret_cast<char*>(data.view), SizeBytes, stream);
        }
    }

    // The C-ABI descriptor of this view, for a call that reads it: work
    // deferred into the buffer is enqueued first (Deferred.hpp).
    tadma_tensor describe() const {
        detail::sync_read(data.ctl);
        return describe_raw();
    }
    // Readable contents: enqueues the work deferred into the buffer.  Needed
    // before reading `data.view` directly (every API call does this itself).
    const Tensor& materialize() const {
        detail::sync_read(data.ctl);
        return *this;
    }
    // The descriptor without synchronising (deferral bookkeeping).
    tadma_tensor describe_raw() const {
        tadma_tensor d{};
        d.data = static_cast<void*>(data.view);
        d.dtype = dtype_v<T>;
        d.rank = (int32_t)Rank;
        for (int i = 0; i < Rank; i++) {
            d.dims[i] = Dims::Arr[i];
            d.strides[i] = Strides::Arr[i];
        }
        return d;
    }

    // ------------------------------------------------------------ views --
    template <typename NewDims, typename NewStrides>
    using View = Tensor<T, Allocator, NewDims, NewStrides>;

    // transpose<D0, D1>: swap two axes (Tensor.hpp:358-364).
    // transpose<P0, ..., Pr-1>: permutation (ONNX Transpose perm).
    // transpose<>: reverse all axes (ONNX default perm).
    template <int... P>
    auto transpose() const {
        if constexpr (sizeof...(P) == 0) {
            return View<SeqFromArray<reversed_arr<Dims>(Dims::Arr)>, SeqFromArray<reversed_arr<Dims>(Strides::Arr)>>(data);
        } else if constexpr (sizeof...(P) == 2) {
            constexpr int p[] = {P...};
            constexpr int D0 = p[0] < 0 ? p[0] + Rank : p[0], D1 = p[1] < 0 ? p[1] + Rank : p[1];
            static_assert(D0 < Rank && D1 < Rank, "Invalid dimensions for transpose");
            return View<typename Dims::template Swap<D0, D1>, typename Strides::template Swap<D0, D1>>(data);
        } else {
            static_assert(sizeof...(P) == Rank, "transpose needs two axes or a full permutation");
            return View<SeqFromArray<permute_arr<Dims, P...>(Dims::Arr)>, SeqFromArray<permute_arr<Dims, P...>(Strides::Arr)>>(data);
        }
    }

    // slice<Start, End, Axis, Step> (Tensor.hpp:295-316): a strided view.
    template <int Start, int End, int Axis = 0, int Step = 1>
    auto slice() const {
        constexpr int DimIndex = Axis < 0 ? Rank + Axis : Axis;
        constexpr int64_t DimSize = Dims::Values(DimIndex);
        constexpr int64_t StartIndex = Start < 0 ? DimSize + Start : (Start > DimSize ? DimSize : Start);
        constexpr int64_t EndIndex = End < 0 ? DimSize + End + 1 : (End > DimSize ? DimSize : End);
        static_assert(StartIndex >= 0 && StartIndex <= DimSize, "Start index out of bounds");
        static_assert(EndIndex >= 0 && EndIndex <= DimSize, "End index out of bounds");
        static_assert(Step != 0, "Step must be non-zero");
        constexpr int64_t Span = Step > 0 ? (EndIndex > StartIndex ? (EndIndex - StartIndex + Step - 1) / Step : 0)
                                          : (StartIndex > EndIndex ? (StartIndex - EndIndex - Step - 1) / (-Step) : 0);
        using NewDims = typename Dims::template Set<DimIndex, Span>;
        using NewStrides = typename Strides::template Set<DimIndex, Strides::Values(DimIndex) * Step>;
        return View<NewDims, NewStrides>(data + Strides::Values(DimIndex) * StartIndex);
    }

    // squeeze<Dims...>: remove the listed extent-1 axes (all of them when none are listed).
    template <int... Ds>
    auto squeeze() const {
        constexpr auto keep = [] {
            std::array<bool, Rank> k{};
            for (int i = 0; i < Rank; i++) k[i] = true;
            if constexpr (sizeof...(Ds) == 0) {
                for (int i = 0; i < Rank; i++)
                    if (Dims::Arr[i] == 1) k[i] = false;
            } else {
                constexpr int ds[] = {Ds...};
                for (int d : ds) k[d < 0 ? d + Rank : d] = false;
            }
            return k;
        }();
        static_assert(((Dims::Values(Ds < 0 ? Ds + Rank : Ds) == 1) && ...), "squeeze of an axis with extent != 1");
        constexpr int n = [&] {
            int c = 0;
            for (bool b : keep) c += b;
            return c;
        }();
        constexpr auto dims = [&] {
            std::array<int64_t, n> a{};
            for (int i = 0, k = 0; i < Rank; i++)
                if (keep[i]) a[k++] = Dims::Arr[i];
            return a;
        }();
        constexpr auto strides = [&] {
            std::array<int64_t, n> a{};
            for (int i = 0, k = 0; i < Rank; i++)
                if (keep[i]) a[k++] = Strides::Arr[i];
            return a;
        }();
        return View<SeqFromArray<dims>, SeqFromArray<strides>>(data);
    }

    // unsqueeze<Dim, Broadcast> (Tensor.hpp:323-331): insert an axis of
    // extent Broadcast with stride 0.
    template <int Dim = -1, int Broadcast = 1>
    auto unsqueeze() const {
        constexpr int DimIndex = Dim < 0 ? Rank + Dim + 1 : Dim;
        static_assert(DimIndex >= 0 && DimIndex <= Rank, "unsqueeze axis out of range");
        return View<typename Dims::template Insert<DimIndex, Broadcast>, typename Strides::template Insert<DimIndex, 0>>(data);
    }

    // broadcast<Dim, Size> (Tensor.hpp:333-336)
    template <int Dim, int NewSize>
    auto broadcast() const {
        static_assert(Dims::Values(Dim) == 1, "broadcast of an axis with extent != 1");
        return View<typename Dims::template Set<Dim, NewSize>, typename Strides::template Set<Dim, 0>>(data);
    }

    template <AnySequence TargetDims>
        requires(broadcastable_to<Dims, Strides, TargetDims>())
    auto broadcastTo() const {
        return View<TargetDims, SeqFromArray<broadcast_strides_arr<Dims, Strides, TargetDims>()>>(data);
    }
    template <AnyTensor U>
    auto broadcastTo(const U&) const {
        return this->template broadcastTo<typename U::Dims>();
    }
    // broadcastTo<TYPE(t)>(): the target given as a tensor type (generated code's Expand).
    template <AnyTensor U>
    auto broadcastTo() const {
        return this->template broadcastTo<typename std::decay_t<U>::Dims>();
    }

    // reshape<Sequence<...>> / reshape<d0, d1, ...> (Tensor.hpp:366-380); one
    // -1 is inferred; a non-contiguous view is materialised first (clone).
    template <AnySequence NewDims>
    auto reshape() const {
        constexpr int in1 = NewDims::template IndexOf<-1>;
        constexpr auto dims = [] {
            auto a = NewDims::Arr;
            if (in1 != -1) {
                int64_t known = 1;
                for (int i = 0; i < NewDims::Size; i++)
                    if (i != in1) known *= a[i];
                a[in1] = known ? Size / known : 0;
            }
            return a;
        }();
        using D = SeqFromArray<dims>;
        static_assert(D::Product() == Size, "reshape must keep the element count");
        if constexpr (!NormalStrides) {
            auto c = clone();
            return Tensor<T, Allocator, D>(c.data);
        } else {
            return Tensor<T, Allocator, D>(data);
        }
    }
    // reshape<d0, d1, ...>, or reshape<shape> with one compile-time shape value
    // (a ConstexprHolder or ConstTensor of Constexpr.hpp, as generated code
    // passes the output of its shape arithmetic).  ONNX Reshape rules: 0
    // copies the input dim at that position, one -1 is inferred.
    template <auto... NewDims>
        requires(sizeof...(NewDims) > 0)
    auto reshape() const {
        constexpr auto req = [] {
            std::array<int64_t, (shape_arg_size<NewDims>() + ...)> r{};
            std::size_t k = 0;
            ((([&] {
                 for (auto v : shape_arg_values<NewDims>()) r[k++] = v;
             })()),
             ...);
            for (std::size_t i = 0; i < r.size(); i++)
                if (r[i] == 0 && (int64_t)i < Rank) r[i] = Dims::Arr[i];
            return r;
        }();
        return this->template reshape<SeqFromArray<req>>();
    }

    // index<Axis>(i): drop Axis at position i (Tensor.hpp:183-187).
    template <int Axis>
    auto index(int64_t i) const {
        static_assert(Axis >= 0 && Axis < Rank);
        return View<typename Dims::template Remove<Axis>, typename Strides::template Remove<Axis>>(data + i * Strides::Values(Axis));
    }

    // split<Axis, Sections> (Tensor.hpp:410-422): a tuple of views.
    template <int Axis, AnySequence Sections>
    auto split() const {
        static_assert(Sections::Sum() == Dims::Values(Axis), "sections must cover the axis");
        return split_impl<Axis, Sections>(std::make_index_sequence<Sections::Size>());
    }

    auto removeFakeDims() const {
        using D = SeqFromArray<fake_free_arr<Dims, Strides, false>()>;
        using S = SeqFromArray<fake_free_arr<Dims, Strides, true>()>;
        return View<D, S>(data);
    }

    // ------------------------------------------------------------- copies --
    auto clone() const;
    auto contiguous() const {
        if constexpr (NormalStrides) return materialize();
        else return clone();
    }
    template <Memory NewDevice>
    auto to() const;
    template <Element U>
    auto to() const;
    template <AnyTensor U>
    void copyTo(U& other) const;

    // --------------------------------------------------------- reductions --
    template <int D, bool KeepDims = true>
    auto sum() const;
    template <int D, bool KeepDims = true>
    auto min() const;
    template <int D, bool KeepDims = true>
    auto max() const;
    template <int D, bool KeepDims = true>
    auto mean() const;
    template <int D, bool KeepDims = false>
    auto argmax() const;
    template <int D, bool KeepDims = false>
    auto argmin() const;

    // ------------------------------------------------------ element access --
    // Host tensors only (a CUDA tensor's elements live on the device).
    template <typename... Is>
        requires(sizeof...(Is) == Rank && device == kCPU)
    T& operator()(Is... is) const {
        const int64_t idx[] = {int64_t(is)..., 0};
        int64_t off = 0;
        for (int i = 0; i < Rank; i++) off += idx[i] * Strides::Arr[i];
        return data.view[off];
    }
    T& operator[](int64_t i) const
        requires(device == kCPU)
    {
        int64_t off = 0;
        for (int d = (int)Rank - 1; d >= 0; d--) {
            off += (i % Dims::Arr[d]) * Strides::Arr[d];
            i /= Dims::Arr[d];
        }
        return data.view[off];
    }
    // Value of a one-element tensor (synchronising read for CUDA tensors).
    T scalar() const
        requires(IsScalar)
    {
        if constexpr (device == kCPU) {
            return data.view[0];
        } else {
            T v;
            detail::sync_read(data.ctl);
            check_cuda(cudaMemcpyAsync(&v, data.view, sizeof(T), cudaMemcpyDeviceToHost, stream));
            check_cuda(cudaStreamSynchronize(stream));
            return v;
        }
    }

  private:
    template <int Axis, AnySequence Sections, std::size_t... I>
    auto split_impl(std::index_sequence<I...>) const {
        constexpr auto offsets = [] {
            std::array<int64_t, Sections::Size> o{};
            int64_t acc = 0;
            for (int i = 0; i < Sections::Size; i++) {
                o[i] = acc;
                acc += Sections::Arr[i];
            }
            return o;
        }();
        return std::make_tuple(
            View<typename Dims::template Set<Axis, Sections::Arr[I]>, Strides>(data + offsets[I] * Strides::Values(Axis))...);
    }
};

template <typename T, typename Dims, typename Strides = Sequence<>>
using CpuTensor = Tensor<T, Allocator<kCPU>, Dims, Strides>;
template <typename T, typename Dims, typename Strides = Sequence<>>
using CudaTensor = Tensor<T, Allocator<kCUDA>, Dims, Strides>;
template <AnyTensor T>
using TensorLike = Tensor<typename T::ValueType, typename T::AllocatorType, typename T::Dims>;
template <AnyTensor T>
using BaseTensor = Tensor<typename T::ValueType, typename T::AllocatorType, typename T::Dims, Sequence<>>;

template <typename A, typename B>
concept Broadcastable = AnyTensor<A> && AnyTensor<B> &&
                        broadcastable_to<typename A::Dims, typename A::Strides, typename B::Dims>();

// ---------------------------------------------------------- copies / casts --

namespace detail {

inline tadma_instr ins(int op, int b = TADMA_SRC_NONE, double imm = 0.0, int round_dtype = -1, int c = TADMA_SRC_NONE) {
    tadma_instr i{};
    i.op = op;
    i.b = b;
    i.c = c;
    i.round_dtype = round_dtype;
    i.imm = imm;
    return i;
}

// out = chain(ins...) on tadma::stream; every input already has out's dims.
// out = chain(ins...) on tadma::stream; every input already has out's dims.
// Deferred (recorded in out's storage, Deferred.hpp) when it can be; else
// launched now, after the buffers' pending work.
template <AnyTensor Out, AnyTensor... In>
void chain(const Out& out, std::initializer_list<tadma_instr> prog, const In&... inputs) {
    static_assert(Out::device == kCUDA && ((In::device == kCUDA) && ...), "tadma ops run on CUDA tensors");
    if (defer_eltwise(out, prog, inputs...)) return;
    sync_write(out.data.ctl);
    tadma_tensor o = out.describe_raw();
    std::array<tadma_tensor, sizeof...(In) + 1> arr{inputs.describe()..., tadma_tensor{}};
    check(tadma_b200_eltwise(&o, arr.data(), (int32_t)sizeof...(In), prog.begin(), (int32_t)prog.size(),
                             TADMA_COMPUTE_AUTO, stream),
          "tadma eltwise");
}

}  // namespace detail

template <typename T, typename A, AnySequence D, AnySequence S>
auto Tensor<T, A, D, S>::clone() const {
    Tensor<T, A, D> result;
    copyTo(result);
    return result;
}

template <typename T, typename A, AnySequence D, AnySequence S>
template <AnyTensor U>
void Tensor<T, A, D, S>::copyTo(U& other) const {
    static_assert(typename U::Dims() == D(), "copyTo needs equal dims");
    using UT = typename U::ValueType;
    if constexpr (device == kCUDA && U::device == kCUDA) {
        detail::chain(other, {detail::ins(TADMA_OP_COPY)}, *this);
    } else if constexpr (U::NormalStrides && NormalStrides && std::is_same_v<UT, T>) {
        cudaMemcpyKind kind = device == kCPU ? (U::device == kCPU ? cudaMemcpyHostToHost : cudaMemcpyHostToDevice)
                                             : cudaMemcpyDeviceToHost;
        detail::sync_read(data.ctl);
        detail::sync_write(other.data.ctl);
        check_cuda(cudaMemcpyAsync(other.data.view, data.view, Size * sizeof(T), kind, stream));
    } else if constexpr (device == kCUDA) {
        auto tmp = this->template to<UT>().contiguous();
        tmp.copyTo(other);
    } else {
        static_assert(device == kCPU && U::device == kCPU, "host <-> device copies need contiguous tensors of one type");
        for (int64_t i = 0; i < Size; i++) other[i] = (UT)(*this)[i];
    }
}

template <typename T, typename A, AnySequence D, AnySequence S>
template <Memory NewDevice>
auto Tensor<T, A, D, S>::to() const {
    if constexpr (NewDevice == device) {
        return *this;
    } else {
        Tensor<T, ::tadma::Allocator<NewDevice>, D> result;
        auto src = contiguous();
        src.copyTo(result);
        if constexpr (NewDevice == kCPU) check_cuda(cudaStreamSynchronize(stream));
        return result;
    }
}

// to<U>: element-type cast (Tensor.hpp:225-228), one COPY chain.
template <typename T, typename A, AnySequence D, AnySequence S>
template <Element U>
auto Tensor<T, A, D, S>::to() const {
    if constexpr (std::is_same_v<U, T>) {
        return *this;
    } else {
        Tensor<U, A, D> result;
        detail::chain(result, {detail::ins(TADMA_OP_COPY)}, *this);
        return result;
    }
}

// ---------------------------------------------------------------- printing --

template <AnyTensor T>
    requires(std::decay_t<T>::device == kCPU)
std::ostream& print_tensor(std::ostream& os, const T& t) {
    using V = typename T::ValueType;
    auto val = [](V v) -> double {
        if constexpr (std::is_same_v<V, __half>) return (double)__half2float(v);
        else if constexpr (std::is_same_v<V, __nv_bfloat16>) return (double)__bfloat162float(v);
        else return (double)v;
    };
    if constexpr (T::Rank == 0) {
        os << val(t.data.view[0]);
    } else {
        std::array<int64_t, T::Rank> idx{};
        for (int64_t e = 0; e < T::Size; e++) {
            int64_t rem = e;
            for (int d = T::Rank - 1; d >= 0; d--) {
                idx[d] = rem % T::Dims::Arr[d];
                rem /= T::Dims::Arr[d];
            }
            int opened = 0;
            for (int d = T::Rank - 1; d >= 0 && idx[d] == 0; d--) opened++;
            for (int k = 0; k < opened; k++) os << '[';
            os << val(t[e]);
            int closed = 0;
            for (int d = T::Rank - 1; d >= 0 && idx[d] == T::Dims::Arr[d] - 1; d--) closed++;
            for (int k = 0; k < closed; k++) os << ']';
            os << (closed == T::Rank ? "\n" : (closed ? ",\n" : ", "));
        }
    }
    return os;
}

template <AnyTensor T>
std::ostream& operator<<(std::ostream& os, const T& t) {
    if constexpr (std::decay_t<T>::device == kCPU) {
        return print_tensor(os, t);
    } else {
        auto host = t.contiguous().template to<kCPU>();
        return print_tensor(os, host);
    }
}

using NoTensor = Tensor<bool, Allocator<kCPU>, Sequence<0>>;

}  // namespace tadma
