// Core.hpp - runtime plumbing of the static-shape Tensor API: memory kinds,
// the thread-local stream, error checks, ref-counted storage and allocators.
//
// Public names follow the reference: Memory {kCPU, kCUDA, kTrampoline}
// (Concepts.hpp:5-9); tadma::stream, init(), deinit(), InitGuard,
// CUDAStreamGuard (Globals.hpp:8-37); check_cuda throwing std::runtime_error
// (Defines.hpp:14-26); HeapStorage (Storage.hpp:16-127); Allocator<kCUDA> with
// stream-ordered cudaMallocAsync / cudaFreeAsync and Allocator<kCPU>
// (Allocator.hpp:18-37).  Every op of the API is asynchronous on
// tadma::stream and runs in libtadma_b200.so (include/tadma_b200.h).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <functional>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../tadma_b200.h"

#ifdef __CUDACC__
#define __multi__ __device__ __host__
#else
#define __multi__
#endif

#ifdef ENABLE_ASSERTS
#include <cassert>
#define ASSERT assert
#else
#define ASSERT(...)
#endif

#define check_cuda(expr)                                                    \
    {                                                                       \
        cudaError_t status__ = (expr);                                      \
        if (status__ != cudaSuccess) throw std::runtime_error(cudaGetErrorString(status__)); \
    }

namespace tadma {

enum Memory { kCPU, kCUDA, kTrampoline };

// Stream every op of the calling thread is enqueued on (reference Globals.hpp:8).
inline thread_local cudaStream_t stream = nullptr;

inline void init() { check_cuda(cudaStreamCreate(&stream)); }

inline void deinit() {
    if (stream) cudaStreamDestroy(stream);
    stream = nullptr;
}

struct InitGuard {
    InitGuard() { init(); }
    ~InitGuard() { deinit(); }
    InitGuard(const InitGuard&) = delete;
    InitGuard& operator=(const InitGuard&) = delete;
};

struct CUDAStreamGuard {
    cudaStream_t oldStream;
    explicit CUDAStreamGuard(cudaStream_t newStream) : oldStream(stream) { stream = newStream; }
    ~CUDAStreamGuard() { stream = oldStream; }
};

namespace detail {
// Library calls made by the header API on this thread (every C-ABI call goes
// through check()); tests read it to count launches.
inline thread_local int64_t calls = 0;

// Turns a C-ABI status into the reference's error convention (std::runtime_error).
inline void check(int rc, const char* what) {
    calls++;
    if (rc != TADMA_OK) throw std::runtime_error(std::string(what) + ": " + tadma_b200_last_error());
}

struct Deferred;

// Control block of an owned buffer: its reference count and deleter, the
// deferred work that will write it (not yet enqueued), and the deferred work
// that reads it (Deferred.hpp).
struct StorageCtl {
    std::atomic<int> refs{1};
    std::function<void()> deleter;
    std::shared_ptr<Deferred> pending;
    std::vector<std::weak_ptr<Deferred>> readers;
};
}  // namespace detail

// Ref-counted pointer on the host side, a raw pointer when copied into a kernel.
template <typename T>
struct HeapStorage {
    using Ctl = detail::StorageCtl;
    T* view = nullptr;
    Ctl* ctl = nullptr;

    HeapStorage() = default;
    HeapStorage(T* p, std::function<void()> deleter) : view(p), ctl(new Ctl) { ctl->deleter = std::move(deleter); }
    explicit HeapStorage(T* p) : view(p) {}  // non-owning
    HeapStorage(const HeapStorage& o) : view(o.view), ctl(o.ctl) {
        if (ctl) ctl->refs++;
    }
    HeapStorage(HeapStorage&& o) noexcept : view(o.view), ctl(o.ctl) {
        o.view = nullptr;
        o.ctl = nullptr;
    }
    HeapStorage& operator=(const HeapStorage& o) {
        if (this != &o) {
            release();
            view = o.view;
            ctl = o.ctl;
            if (ctl) ctl->refs++;
        }
        return *this;
    }
    HeapStorage& operator=(HeapStorage&& o) noexcept {
        if (this != &o) {
            release();
            view = o.view;
            ctl = o.ctl;
            o.view = nullptr;
            o.ctl = nullptr;
        }
        return *this;
    }
    ~HeapStorage() { release(); }

    void release() noexcept {
        if (ctl && --ctl->refs == 0) {
            // Work deferred into a buffer nobody holds any more is dropped
            // unrun; the buffer is freed behind everything already enqueued.
            ctl->pending.reset();
            if (ctl->deleter) ctl->deleter();
            delete ctl;
        }
        ctl = nullptr;
    }
    // Storage acts as a pointer: views share ownership at an element offset.
    HeapStorage operator+(int64_t offset) const {
        HeapStorage s(*this);
        s.view += offset;
        return s;
    }
    T& operator[](int64_t i) const { return view[i]; }
    int use_count() const { return ctl ? ctl->refs.load() : 0; }
};

template <Memory device>
struct Allocator;

template <>
struct Allocator<kCUDA> {
    static constexpr Memory device = kCUDA;
    template <typename T, int64_t Count>
    static HeapStorage<T> allocate() {
        if constexpr (Count == 0) {
            return HeapStorage<T>();
        } else {
            T* ptr = nullptr;
            cudaStream_t s = stream;
            // TADMA_B200_FAIL_ALLOC=1 fails every allocation as an exhausted
            // device would, before any CUDA call (host-side fault injection).
            if (const char* inject = std::getenv("TADMA_B200_FAIL_ALLOC"); inject && inject[0] == '1')
                check_cuda(cudaErrorMemoryAllocation);
            check_cuda(cudaMallocAsync(reinterpret_cast<void**>(&ptr), sizeof(T) * Count, s));
            return HeapStorage<T>(ptr, [ptr, s]() { cudaFreeAsync(ptr, s); });
        }
    }
};

template <>
struct Allocator<kCPU> {
    static constexpr Memory device = kCPU;
    template <typename T, int64_t Count>
    static HeapStorage<T> allocate() {
        if constexpr (Count == 0) {
            return HeapStorage<T>();
        } else {
            T* ptr = new T[Count]();
            return HeapStorage<T>(ptr, [ptr]() { delete[] ptr; });
        }
    }
};

// A tensor with no memory: its value lives in a register of the thread that
// computes it (ExecutionTape::Optimize; the reference's Allocator<kTrampoline>,
// Allocator.hpp:39-44, and TrampolineStorage, Storage.hpp:131-148).
template <>
struct Allocator<kTrampoline> {
    static constexpr Memory device = kTrampoline;
    template <typename T, int64_t Count>
    static HeapStorage<T> allocate() {
        return HeapStorage<T>();
    }
};

template <typename T>
concept AnyAllocator = requires { T::device; };

}  // namespace tadma
