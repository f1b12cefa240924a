// common.cuh - shared device/host helpers of the tadma_b200 kernels (sm_100a).
//
// * dtype traits and scalar conversions (round-to-nearest-even, saturating
//   float->int with NaN -> 0, i.e. the PTX cvt.rzi rule);
// * DivMod: exact 64-bit division by a run-time invariant divisor
//   (Granlund & Montgomery, "Division by invariant integers using
//   multiplication", PLDI 1994, Fig. 4.1) so per-element index math is a
//   multiply-high instead of a 64-bit divide;
// * 16-byte vector load/store helpers with streaming cache hints;
// * host-side error plumbing for the C ABI (thread-local last-error text).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/tadma_b200.h"

namespace tadma_b200 {

// ------------------------------------------------------------------ dtypes --

__host__ __device__ inline int dtype_size(int dt) {
    switch (dt) {
    case TADMA_F32: case TADMA_I32: return 4;
    case TADMA_F16: case TADMA_BF16: return 2;
    case TADMA_F64: case TADMA_I64: return 8;
    case TADMA_U8: case TADMA_BOOL: case TADMA_I8: return 1;
    default: return 0;
    }
}

__host__ __device__ inline bool dtype_is_float(int dt) {
    return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16 || dt == TADMA_F64;
}

// --------------------------------------------------------- scalar convert --

// float -> int64 truncating, saturating, NaN -> 0 (cvt.rzi.s64.f32 semantics).
__device__ __forceinline__ int64_t f2i(float v) { return __float2ll_rz(v); }
__device__ __forceinline__ int64_t f2i(double v) { return __double2ll_rz(v); }

// Load one element of run-time dtype `dt` as compute type C.
template <typename C>
__device__ __forceinline__ C load_as(const char* p, int dt, int64_t off);

template <>
__device__ __forceinline__ float load_as<float>(const char* p, int dt, int64_t off) {
    switch (dt) {
    case TADMA_F32: return reinterpret_cast<const float*>(p)[off];
    case TADMA_F16: return __half2float(reinterpret_cast<const __half*>(p)[off]);
    case TADMA_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off]);
    case TADMA_F64: return __double2float_rn(reinterpret_cast<const double*>(p)[off]);
    case TADMA_I64: return __ll2float_rn(reinterpret_cast<const long long*>(p)[off]);
    case TADMA_I32: return __int2float_rn(reinterpret_cast<const int32_t*>(p)[off]);
    case TADMA_U8: return (float)reinterpret_cast<const uint8_t*>(p)[off];
    case TADMA_BOOL: return reinterpret_cast<const uint8_t*>(p)[off] != 0 ? 1.0f : 0.0f;
    case TADMA_I8: return (float)reinterpret_cast<const int8_t*>(p)[off];
    }
    return 0.0f;
}

template <>
__device__ __forceinline__ double load_as<double>(const char* p, int dt, int64_t off) {
    switch (dt) {
    case TADMA_F32: return (double)reinterpret_cast<const float*>(p)[off];
    case TADMA_F16: return (double)__half2float(reinterpret_cast<const __half*>(p)[off]);
    case TADMA_BF16: return (double)__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off]);
    case TADMA_F64: return reinterpret_cast<const double*>(p)[off];
    case TADMA_I64: return __ll2double_rn(reinterpret_cast<const long long*>(p)[off]);
    case TADMA_I32: return (double)reinterpret_cast<const int32_t*>(p)[off];
    case TADMA_U8: return (double)reinterpret_cast<const uint8_t*>(p)[off];
    case TADMA_BOOL: return reinterpret_cast<const uint8_t*>(p)[off] != 0 ? 1.0 : 0.0;
    case TADMA_I8: return (double)reinterpret_cast<const int8_t*>(p)[off];
    }
    return 0.0;
}

template <>
__device__ __forceinline__ int64_t load_as<int64_t>(const char* p, int dt, int64_t off) {
    switch (dt) {
    case TADMA_F32: return f2i(reinterpret_cast<const float*>(p)[off]);
    case TADMA_F16: return f2i(__half2float(reinterpret_cast<const __half*>(p)[off]));
    case TADMA_BF16: return f2i(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off]));
    case TADMA_F64: return f2i(reinterpret_cast<const double*>(p)[off]);
    case TADMA_I64: return reinterpret_cast<const long long*>(p)[off];
    case TADMA_I32: return reinterpret_cast<const int32_t*>(p)[off];
    case TADMA_U8: return reinterpret_cast<const uint8_t*>(p)[off];
    case TADMA_BOOL: return reinterpret_cast<const uint8_t*>(p)[off] != 0;
    case TADMA_I8: return reinterpret_cast<const int8_t*>(p)[off];
    }
    return 0;
}

// One rounding from double / int64 to a 16-bit float (no detour through
// fp32, which could round twice).  A NaN keeps the bits of the fp32 path.
__device__ __forceinline__ __half d2h(double v) { return v != v ? __float2half_rn(__double2float_rn(v)) : __double2half(v); }
__device__ __forceinline__ __nv_bfloat16 d2bf(double v) {
    return v != v ? __float2bfloat16_rn(__double2float_rn(v)) : __double2bfloat16(v);
}

// Store compute value into element `off` of run-time dtype `dt`, rounded once.
__device__ __forceinline__ void store_from(char* p, int dt, int64_t off, float v) {
    switch (dt) {
    case TADMA_F32: reinterpret_cast<float*>(p)[off] = v; break;
    case TADMA_F16: reinterpret_cast<__half*>(p)[off] = __float2half_rn(v); break;
    case TADMA_BF16: reinterpret_cast<__nv_bfloat16*>(p)[off] = __float2bfloat16_rn(v); break;
    case TADMA_F64: reinterpret_cast<double*>(p)[off] = (double)v; break;
    case TADMA_I64: reinterpret_cast<long long*>(p)[off] = f2i(v); break;
    case TADMA_I32: reinterpret_cast<int32_t*>(p)[off] = (int32_t)f2i(v); break;
    case TADMA_U8: reinterpret_cast<uint8_t*>(p)[off] = (uint8_t)f2i(v); break;
    case TADMA_BOOL: reinterpret_cast<uint8_t*>(p)[off] = v != 0.0f; break;
    case TADMA_I8: reinterpret_cast<int8_t*>(p)[off] = (int8_t)f2i(v); break;
    }
}

__device__ __forceinline__ void store_from(char* p, int dt, int64_t off, double v) {
    switch (dt) {
    case TADMA_F32: reinterpret_cast<float*>(p)[off] = __double2float_rn(v); break;
    case TADMA_F16: reinterpret_cast<__half*>(p)[off] = d2h(v); break;
    case TADMA_BF16: reinterpret_cast<__nv_bfloat16*>(p)[off] = d2bf(v); break;
    case TADMA_F64: reinterpret_cast<double*>(p)[off] = v; break;
    case TADMA_I64: reinterpret_cast<long long*>(p)[off] = f2i(v); break;
    case TADMA_I32: reinterpret_cast<int32_t*>(p)[off] = (int32_t)f2i(v); break;
    case TADMA_U8: reinterpret_cast<uint8_t*>(p)[off] = (uint8_t)f2i(v); break;
    case TADMA_BOOL: reinterpret_cast<uint8_t*>(p)[off] = v != 0.0; break;
    case TADMA_I8: reinterpret_cast<int8_t*>(p)[off] = (int8_t)f2i(v); break;
    }
}

__device__ __forceinline__ void store_from(char* p, int dt, int64_t off, int64_t v) {
    switch (dt) {
    case TADMA_F32: reinterpret_cast<float*>(p)[off] = __ll2float_rn(v); break;
    case TADMA_F16: reinterpret_cast<__half*>(p)[off] = __ll2half_rn(v); break;
    case TADMA_BF16: reinterpret_cast<__nv_bfloat16*>(p)[off] = __ll2bfloat16_rn(v); break;
    case TADMA_F64: reinterpret_cast<double*>(p)[off] = __ll2double_rn(v); break;
    case TADMA_I64: reinterpret_cast<long long*>(p)[off] = v; break;
    case TADMA_I32: reinterpret_cast<int32_t*>(p)[off] = (int32_t)v; break;
    case TADMA_U8: reinterpret_cast<uint8_t*>(p)[off] = (uint8_t)v; break;
    case TADMA_BOOL: reinterpret_cast<uint8_t*>(p)[off] = v != 0; break;
    case TADMA_I8: reinterpret_cast<int8_t*>(p)[off] = (int8_t)v; break;
    }
}

// Value a tensor of dtype `dt` would hold for v (materialised intermediate).
__device__ __forceinline__ float round_to(float v, int dt) {
    switch (dt) {
    case TADMA_F16: return __half2float(__float2half_rn(v));
    case TADMA_BF16: return __bfloat162float(__float2bfloat16_rn(v));
    case TADMA_F32: case TADMA_F64: return v;
    case TADMA_I64: return __ll2float_rn(f2i(v));
    case TADMA_I32: return (float)(int32_t)f2i(v);
    case TADMA_U8: return (float)(uint8_t)f2i(v);
    case TADMA_BOOL: return v != 0.0f ? 1.0f : 0.0f;
    case TADMA_I8: return (float)(int8_t)f2i(v);
    }
    return v;
}

__device__ __forceinline__ double round_to(double v, int dt) {
    switch (dt) {
    case TADMA_F32: return (double)__double2float_rn(v);
    case TADMA_F16: return (double)__half2float(d2h(v));
    case TADMA_BF16: return (double)__bfloat162float(d2bf(v));
    case TADMA_F64: return v;
    case TADMA_I64: return __ll2double_rn(f2i(v));
    case TADMA_I32: return (double)(int32_t)f2i(v);
    case TADMA_U8: return (double)(uint8_t)f2i(v);
    case TADMA_BOOL: return v != 0.0 ? 1.0 : 0.0;
    case TADMA_I8: return (double)(int8_t)f2i(v);
    }
    return v;
}

__device__ __forceinline__ int64_t round_to(int64_t v, int dt) {
    switch (dt) {
    case TADMA_I32: return (int32_t)v;
    case TADMA_U8: return (uint8_t)v;
    case TADMA_BOOL: return v != 0;
    case TADMA_I8: return (int8_t)v;
    case TADMA_F32: return f2i(__ll2float_rn(v));
    case TADMA_F16: return f2i(__half2float(__ll2half_rn(v)));
    case TADMA_BF16: return f2i(__bfloat162float(__ll2bfloat16_rn(v)));
    case TADMA_F64: return f2i(__ll2double_rn(v));
    }
    return v;
}

// ------------------------------------------------------------------ DivMod --

// Exact floor(n / d) for every 64-bit n, d >= 1 (GM94 Fig. 4.1 with N = 64).
struct DivMod {
    uint64_t d = 1;
    uint64_t m = 0;    // magic multiplier, 64-bit dividends
    uint32_t m32 = 0;  // magic multiplier, dividends below 2^32 (0 when d >= 2^32)
    uint16_t s1 = 0;   // min(l, 1)
    uint16_t s2 = 0;   // max(l - 1, 0)

    DivMod() = default;
    __host__ explicit DivMod(uint64_t d_) : d(d_ ? d_ : 1) {
        uint32_t l = 0;
        while (l < 64 && ((unsigned __int128)1 << l) < d) l++;  // l = ceil(log2 d)
        unsigned __int128 two64 = (unsigned __int128)1 << 64;
        unsigned __int128 num = two64 * (((unsigned __int128)1 << l) - d);
        m = (uint64_t)(num / d + 1);
        // The same construction at N = 32 (2^l - d < d, so the quotient fits).
        if (d <= 0xffffffffull) m32 = (uint32_t)((((uint64_t)1 << 32) * (((uint64_t)1 << l) - d)) / d + 1);
        s1 = (uint16_t)(l < 1 ? l : 1);
        s2 = (uint16_t)(l > 0 ? l - 1 : 0);
    }
    // n / d for n < 2^32 and d < 2^32: one 32-bit high multiply instead of
    // the 64-bit one (several IMADs and carries on the GPU).
    __host__ __device__ __forceinline__ uint32_t div32(uint32_t n) const {
#ifdef __CUDA_ARCH__
        uint32_t t1 = __umulhi(m32, n);
#else
        uint32_t t1 = (uint32_t)(((uint64_t)m32 * n) >> 32);
#endif
        return (t1 + ((n - t1) >> s1)) >> s2;
    }
    __host__ __device__ __forceinline__ uint64_t div(uint64_t n) const {
#ifdef __CUDA_ARCH__
        uint64_t t1 = __umul64hi(m, n);
#else
        uint64_t t1 = (uint64_t)(((unsigned __int128)m * n) >> 64);
#endif
        return (t1 + ((n - t1) >> s1)) >> s2;
    }
    __host__ __device__ __forceinline__ void divmod(uint64_t n, uint64_t& q, uint64_t& r) const {
        q = div(n);
        r = n - q * d;
    }
};

// ---------------------------------------------------------- vector memory --

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }

// Asynchronous 16-byte global -> shared copies (cp.async, L2-only): the
// issuing thread's groups complete in order; cp.async.wait_group N waits
// until at most N of its groups are still in flight (a hardware wait).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint4 ld_v4(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ void st_stream_v4(void* p, uint4 v) { __stcs(reinterpret_cast<uint4*>(p), v); }

// L2 eviction-priority policies (PTX createpolicy) for loads whose reuse is
// known: evict_last keeps a small operand that every row re-reads (e.g. a
// position table) resident while a large stream passes through L2;
// evict_first marks data read once.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint4 ld_nc_v4_policy(const void* p, uint64_t pol) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(pol));
    return r;
}
__device__ __forceinline__ void st_v4(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// Unpack / pack 8 x 16-bit floats <-> 8 x fp32.
__device__ __forceinline__ void unpack8(uint4 r, int dt, float* f) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if (dt == TADMA_BF16) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            float2 t = __half22float2(h);
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
}

__device__ __forceinline__ uint4 pack8(const float* f, int dt) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if (dt == TADMA_BF16) {
            __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&b);
        } else {
            __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// ------------------------------------------------------------- reductions --

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        T w = __shfl_xor_sync(0xffffffffu, v, o);
        v = (w > v || w != w) ? w : v;
    }
    return v;
}

// Programmatic dependent launch (sm_90+).  A kernel launched with
// launch_pdl() may be scheduled while the previous kernel of its stream is
// still running: it lets its own dependents launch at once
// (griddepcontrol.launch_dependents) and waits for the previous grid to
// complete and flush its writes (griddepcontrol.wait) before it touches
// global memory.  Launched normally, both instructions are no-ops.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// 2^x on the SFU (ex2.approx.ftz: max relative error ~2^-22).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Packed fp32x2 arithmetic (sm_100): two lanes per instruction, each lane
// rounded exactly like the scalar op (__fmul_rn / __fadd_rn / fmaf).
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// max / min that return NaN when either input is NaN (PTX max.NaN / min.NaN,
// one ALU op): the "NaN sticks once seen" rule of the max/min reductions.
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float fmin_nan(float a, float b) {
    float r;
    asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// ------------------------------------------------------------- host side --

// Launches kernel<<<grid, block, smem, stream>>>(args...) with programmatic
// stream serialisation, so its CTAs can be scheduled during the previous
// kernel's tail; the kernel must call pdl_begin() before any global access.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Per-thread last error message (tadma_b200_last_error).
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);
// Stream-ordered device workspace (cudaMallocAsync).  With TADMA_B200_FAIL_ALLOC=1
// in the environment every call fails as on an exhausted device
// (cudaErrorMemoryAllocation) without calling CUDA: host-side fault injection
// for tests of the error path.
cudaError_t workspace_alloc(void** p, size_t bytes, cudaStream_t s);
// SM count of the current device (cached per device).
int sm_count();
// Validates a tensor descriptor; returns "" or a message.
std::string check_tensor(const tadma_tensor* t, const char* name, bool need_data = true);
int64_t numel(const tadma_tensor* t);

}  // namespace tadma_b200
