// norm.cu - fused reduce-then-broadcast row kernels (sm_100a): softmax,
// LayerNorm (ONNX and TADMA eps placement) and RMSNorm.
//
// The reference composes these from separate kernels, every intermediate a
// full tensor in HBM:
// * softmax (Operations.hpp:190-193): exp node, sum ReduceKernel, in-place
//   divide node -> 3 reads + 2 writes of the data, and no max subtraction
//   (fp16 exp overflows for x > ~11);
// * layer_norm (Operations.hpp:195-220): mean reduce, squared-difference
//   node, sqrt-post reduce, normalise node -> ~5 passes;
// * rms_norm (Operations.hpp:222-233): square-pre reduce, divide node.
//
// Here a row of up to 32 lanes x 8 chunks x 16 bytes (2048 fp16/bf16 or
// 1024 fp32 elements) lives in one warp's registers: one 16-byte-vector
// read, the statistics by shuffle butterflies, one write.  Softmax subtracts
// the row max (same value in exact arithmetic, no overflow).  Longer or
// strided rows take a block-per-row kernel that re-reads the row (L2-hot).
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"
#include "layout.hpp"

namespace tadma_b200 {

namespace {

enum Mode { M_SOFTMAX = 0, M_LN_ONNX = 1, M_LN_TADMA = 2, M_RMS = 3 };

constexpr int THREADS = 256;

struct NormParams {
    const char* in;
    char* out;
    const char* gamma;
    const char* beta;
    int32_t dtype, out_dtype, g_dtype, b_dtype;
    int32_t gb_vec;  // gamma/beta have x's dtype, stride 1, 16-byte aligned
    int32_t mode;
    float eps;
    int32_t pad;
    int64_t nrows, L;
    int64_t in_row_stride, out_row_stride;
    int64_t in_ax_stride, out_ax_stride;
    int64_t g_stride, b_stride;
    // folded row dims (block kernel)
    int32_t krank, pad2;
    DivMod kdm[TADMA_MAX_RANK];
    int64_t kin[TADMA_MAX_RANK];
    int64_t kout[TADMA_MAX_RANK];
};

template <typename T>
struct VecT;
template <>
struct VecT<float> {
    static constexpr int N = 4;
    static constexpr int DT = TADMA_F32;
};
template <>
struct VecT<__half> {
    static constexpr int N = 8;
    static constexpr int DT = TADMA_F16;
};
template <>
struct VecT<__nv_bfloat16> {
    static constexpr int N = 8;
    static constexpr int DT = TADMA_BF16;
};

template <typename T>
__device__ __forceinline__ void cvt_in(uint4 r, float* f) {
    if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(r.x);
        f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z);
        f[3] = __uint_as_float(r.w);
    } else {
        unpack8(r, VecT<T>::DT, f);
    }
}

template <typename T>
__device__ __forceinline__ uint4 cvt_out(const float* f) {
    if constexpr (sizeof(T) == 4) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
    } else {
        return pack8(f, VecT<T>::DT);
    }
}

// N elements of a strided operand of run-time dtype as fp32, the dtype
// dispatched once for all N (per-element gamma / beta layouts).
template <int N>
__device__ __forceinline__ void load_strided(const char* p, int dt, int64_t off, int64_t stride, float (&f)[N]) {
    switch (dt) {
    case TADMA_F32:
#pragma unroll
        for (int j = 0; j < N; j++) f[j] = reinterpret_cast<const float*>(p)[off + j * stride];
        break;
    case TADMA_F16:
#pragma unroll
        for (int j = 0; j < N; j++) f[j] = __half2float(reinterpret_cast<const __half*>(p)[off + j * stride]);
        break;
    case TADMA_BF16:
#pragma unroll
        for (int j = 0; j < N; j++) f[j] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off + j * stride]);
        break;
    default:
#pragma unroll
        for (int j = 0; j < N; j++) f[j] = load_as<float>(p, dt, off + j * stride);
        break;
    }
}

template <typename T>
__device__ __forceinline__ float fast_exp(float x) {
    // 16-bit outputs: the fast exponential's few-ulp fp32 error is far below
    // half an fp16/bf16 ulp; fp32 outputs use the accurate expf.
    if constexpr (sizeof(T) == 4) return expf(x);
    else return __expf(x);
}

// ----------------------------------------------------------- warp kernels --

// Statistics, normalisation and store of one row held in a warp's registers
// (lane l holds chunks c * 32 + l, N elements each; chunks past L hold the
// neutral value of the mode).
// Two 16-bit values (one 32-bit word, low half first) widened to fp32x2.
template <typename T>
__device__ __forceinline__ unsigned long long widen2(uint32_t w) {
    if constexpr (std::is_same<T, __half>::value) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
        return f2_pack(f.x, f.y);
    } else {
        return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
}

// 16-bit rows: the same statistics with the element arithmetic on packed
// fp32x2 instructions (two elements per instruction, each rounded like the
// scalar op), the softmax exponent folded into one fused multiply-add:
//   softmax   e = 2^(x log2e - m log2e),  y = e * (1 / sum e)
//   LayerNorm y = ((x - mean) * rstd) * gamma + beta  (x - mean first, so a
//             value equal to the mean gives exactly 0, as the reference does)
//   RMSNorm   y = x * (1 / sqrt(mean(x^2) + eps))
// Outputs are 16-bit, so the reassociation stays far inside half an ulp.
template <typename T, int CH, int MODE>
__device__ __forceinline__ void rownorm_finish_packed(float (&v)[CH][VecT<T>::N], const NormParams& p, int lane, T* y) {
    constexpr int BM = MODE & 3;          // softmax / LN ONNX / LN TADMA / RMS
    constexpr bool GBV = (MODE & 4) == 0;  // gamma/beta: x dtype, stride 1, 16-byte aligned
    constexpr int N = VecT<T>::N;
    constexpr int H = N / 2;
    typedef unsigned long long u64;
    const float fL = (float)p.L;
    if constexpr (BM == M_SOFTMAX) {
        float m = -INFINITY;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) m = fmaxf(m, v[c][j]);
        m = warp_max(m);
        constexpr float L2E = 1.4426950408889634f;
        const u64 k2 = f2_pack(L2E, L2E), nm2 = f2_pack(-m * L2E, -m * L2E);
        u64 s2 = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int h = 0; h < H; h++) {
                float a, b;
                f2_unpack(f2_fma(f2_pack(v[c][2 * h], v[c][2 * h + 1]), k2, nm2), a, b);
                a = ex2_approx(a);
                b = ex2_approx(b);
                // chunks past L hold -inf: 2^-inf = 0 adds nothing
                v[c][2 * h] = a;
                v[c][2 * h + 1] = b;
                s2 = f2_add(s2, f2_pack(a, b));
            }
        float s0, s1;
        f2_unpack(s2, s0, s1);
        const float inv = 1.0f / warp_sum(s0 + s1);
        const u64 i2 = f2_pack(inv, inv);
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int h = 0; h < H; h++) f2_unpack(f2_mul(f2_pack(v[c][2 * h], v[c][2 * h + 1]), i2), v[c][2 * h], v[c][2 * h + 1]);
    } else if constexpr (BM == M_RMS) {
        u64 q2 = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int h = 0; h < H; h++) {
                const u64 x = f2_pack(v[c][2 * h], v[c][2 * h + 1]);
                q2 = f2_fma(x, x, q2);
            }
        float q0, q1;
        f2_unpack(q2, q0, q1);
        const float r = 1.0f / sqrtf(warp_sum(q0 + q1) / fL + p.eps);
        const u64 r2 = f2_pack(r, r);
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int h = 0; h < H; h++) f2_unpack(f2_mul(f2_pack(v[c][2 * h], v[c][2 * h + 1]), r2), v[c][2 * h], v[c][2 * h + 1]);
    } else {
        u64 s2 = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int h = 0; h < H; h++) s2 = f2_add(s2, f2_pack(v[c][2 * h], v[c][2 * h + 1]));
        float s0, s1;
        f2_unpack(s2, s0, s1);
        const float mean = warp_sum(s0 + s1) / fL;
        const u64 nmean2 = f2_pack(-mean, -mean);
        u64 q2 = f2_pack(0.0f, 0.0f);
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t col = ((int64_t)c * 32 + lane) * N;
            if (col < p.L) {
#pragma unroll
                for (int h = 0; h < H; h++) {
                    const u64 d = f2_add(f2_pack(v[c][2 * h], v[c][2 * h + 1]), nmean2);
                    q2 = f2_fma(d, d, q2);
                }
            }
        }
        float q0, q1;
        f2_unpack(q2, q0, q1);
        const float var = warp_sum(q0 + q1) / fL;
        const float rstd = (BM == M_LN_ONNX) ? 1.0f / sqrtf(var + p.eps) : 1.0f / (sqrtf(var) + p.eps);
        const u64 r2 = f2_pack(rstd, rstd);
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t col = ((int64_t)c * 32 + lane) * N;
            if (col < p.L) {
                if constexpr (GBV) {
                    // gamma / beta stay raw (4 registers each) and are widened
                    // a pair at a time
                    uint4 gr = make_uint4(0, 0, 0, 0), br = make_uint4(0, 0, 0, 0);
                    if (p.gamma) gr = ld_nc_v4(reinterpret_cast<const T*>(p.gamma) + col);
                    if (p.beta) br = ld_nc_v4(reinterpret_cast<const T*>(p.beta) + col);
                    const uint32_t gw[4] = {gr.x, gr.y, gr.z, gr.w}, bw[4] = {br.x, br.y, br.z, br.w};
#pragma unroll
                    for (int h = 0; h < H; h++) {
                        u64 t = f2_mul(f2_add(f2_pack(v[c][2 * h], v[c][2 * h + 1]), nmean2), r2);
                        if (p.gamma && p.beta) t = f2_fma(t, widen2<T>(gw[h]), widen2<T>(bw[h]));
                        else if (p.gamma) t = f2_mul(t, widen2<T>(gw[h]));
                        else if (p.beta) t = f2_add(t, widen2<T>(bw[h]));
                        f2_unpack(t, v[c][2 * h], v[c][2 * h + 1]);
                    }
                } else {
                    // a pair of gamma / beta values at a time keeps 4 registers live
#pragma unroll
                    for (int h = 0; h < H; h++) {
                        float g[2], b[2];
                        if (p.gamma) load_strided<2>(p.gamma, p.g_dtype, (col + 2 * h) * p.g_stride, p.g_stride, g);
                        if (p.beta) load_strided<2>(p.beta, p.b_dtype, (col + 2 * h) * p.b_stride, p.b_stride, b);
#pragma unroll
                        for (int k = 0; k < 2; k++) {
                            float t = (v[c][2 * h + k] - mean) * rstd;
                            if (p.gamma) t = t * g[k];
                            if (p.beta) t = t + b[k];
                            v[c][2 * h + k] = t;
                        }
                    }
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < CH; c++) {
        const int64_t col = ((int64_t)c * 32 + lane) * N;
        if (col < p.L) st_stream_v4(y + col, cvt_out<T>(v[c]));
    }
}

template <typename T, int CH, int MODE>
__device__ __forceinline__ void rownorm_finish(float (&v)[CH][VecT<T>::N], const NormParams& p, int lane, T* y) {
    constexpr int BM = MODE & 3;          // softmax / LN ONNX / LN TADMA / RMS
    constexpr bool GBV = (MODE & 4) == 0;  // gamma/beta: x dtype, stride 1, 16-byte aligned
    if constexpr (sizeof(T) == 2) {
        rownorm_finish_packed<T, CH, MODE>(v, p, lane, y);
        return;
    }
    constexpr int N = VecT<T>::N;
    const float fL = (float)p.L;
    if constexpr (BM == M_SOFTMAX) {
        float m = -INFINITY;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) m = fmaxf(m, v[c][j]);
        m = warp_max(m);
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) {
                v[c][j] = fast_exp<T>(v[c][j] - m);
                s += v[c][j];
            }
        s = warp_sum(s);
        const float inv = 1.0f / s;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) v[c][j] *= inv;
    } else if constexpr (BM == M_RMS) {
        float ss = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) ss += v[c][j] * v[c][j];
        ss = warp_sum(ss);
        const float r = 1.0f / sqrtf(ss / fL + p.eps);
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) v[c][j] *= r;
    } else {
        float sum = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; c++)
#pragma unroll
            for (int j = 0; j < N; j++) sum += v[c][j];
        const float mean = warp_sum(sum) / fL;
        float sq = 0.0f;
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t col = ((int64_t)c * 32 + lane) * N;
            if (col < p.L) {
#pragma unroll
                for (int j = 0; j < N; j++) {
                    const float d = v[c][j] - mean;
                    sq += d * d;
                }
            }
        }
        const float var = warp_sum(sq) / fL;
        const float rstd = (BM == M_LN_ONNX) ? 1.0f / sqrtf(var + p.eps) : 1.0f / (sqrtf(var) + p.eps);
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t col = ((int64_t)c * 32 + lane) * N;
            if (col < p.L) {
                float g[N], b[N];
                if constexpr (GBV) {
                    // raw 16-byte loads converted at use keep few registers live
                    if (p.gamma) cvt_in<T>(ld_nc_v4(reinterpret_cast<const T*>(p.gamma) + col), g);
                    if (p.beta) cvt_in<T>(ld_nc_v4(reinterpret_cast<const T*>(p.beta) + col), b);
                } else {
                    if (p.gamma) load_strided<N>(p.gamma, p.g_dtype, col * p.g_stride, p.g_stride, g);
                    if (p.beta) load_strided<N>(p.beta, p.b_dtype, col * p.b_stride, p.b_stride, b);
                }
#pragma unroll
                for (int j = 0; j < N; j++) {
                    float t = (v[c][j] - mean) * rstd;
                    if (p.gamma) t = t * g[j];
                    if (p.beta) t = t + b[j];
                    v[c][j] = t;
                }
            }
        }
    }
#pragma unroll
    for (int c = 0; c < CH; c++) {
        const int64_t col = ((int64_t)c * 32 + lane) * N;
        if (col < p.L) st_stream_v4(y + col, cvt_out<T>(v[c]));
    }
}

// Resident CTAs per SM the register cap aims for.  16-bit rows of <= 4 chunks
// per lane are latency-bound: fp16 rows fit 4 CTAs (64 registers) without
// spills, bf16 rows 3 (their widening keeps more values live); 8-chunk and
// fp32 rows keep their registers (2 CTAs per SM).
template <typename T, int CH>
constexpr int norm_min_blocks() {
    if (CH > 4 || sizeof(T) == 4) return 2;
    return std::is_same<T, __half>::value ? 4 : 3;
}
template <typename T, int CH, int MODE>
__global__ void __launch_bounds__(THREADS, norm_min_blocks<T, CH>()) rownorm_warp_kernel(const __grid_constant__ NormParams p) {
    pdl_begin();
    constexpr int N = VecT<T>::N;
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    for (int64_t row = gw; row < p.nrows; row += nw) {
        const T* x = reinterpret_cast<const T*>(p.in) + row * p.in_row_stride;
        float v[CH][N];
#pragma unroll
        for (int c = 0; c < CH; c++) {
            const int64_t col = ((int64_t)c * 32 + lane) * N;
            if (col < p.L) {
                cvt_in<T>(ld_stream_v4(x + col), v[c]);
            } else {
#pragma unroll
                for (int j = 0; j < N; j++) v[c][j] = ((MODE & 3) == M_SOFTMAX) ? -INFINITY : 0.0f;
            }
        }
        rownorm_finish<T, CH, MODE>(v, p, lane, reinterpret_cast<T*>(p.out) + row * p.out_row_stride);
    }
}

// ---------------------------------------------------------- block kernel --
// One CTA per row, any axis stride and dtype; re-reads the row per pass.

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
    v = is_max ? warp_max(v) : warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    float r = sh[0];
    for (int i = 1; i < THREADS / 32; i++) r = is_max ? fmaxf(r, sh[i]) : r + sh[i];
    return r;
}

__global__ void __launch_bounds__(THREADS) rownorm_block_kernel(const __grid_constant__ NormParams p) {
    pdl_begin();
    __shared__ float sh[THREADS / 32];
    for (int64_t row = blockIdx.x; row < p.nrows; row += gridDim.x) {
        uint64_t e = (uint64_t)row;
        int64_t ib = 0, ob = 0;
        for (int d = p.krank - 1; d >= 1; d--) {
            uint64_t q, r;
            p.kdm[d].divmod(e, q, r);
            ib += (int64_t)r * p.kin[d];
            ob += (int64_t)r * p.kout[d];
            e = q;
        }
        ib += (int64_t)e * p.kin[0];
        ob += (int64_t)e * p.kout[0];
        const float fL = (float)p.L;
        float a = 0.0f, b = 0.0f;
        if (p.mode == M_SOFTMAX) {
            float m = -INFINITY;
            for (int64_t i = threadIdx.x; i < p.L; i += THREADS) m = fmaxf(m, load_as<float>(p.in, p.dtype, ib + i * p.in_ax_stride));
            a = block_reduce(m, true, sh);
            float s = 0.0f;
            for (int64_t i = threadIdx.x; i < p.L; i += THREADS) s += expf(load_as<float>(p.in, p.dtype, ib + i * p.in_ax_stride) - a);
            b = 1.0f / block_reduce(s, false, sh);
        } else if (p.mode == M_RMS) {
            float ss = 0.0f;
            for (int64_t i = threadIdx.x; i < p.L; i += THREADS) {
                float v = load_as<float>(p.in, p.dtype, ib + i * p.in_ax_stride);
                ss += v * v;
            }
            b = 1.0f / sqrtf(block_reduce(ss, false, sh) / fL + p.eps);
        } else {
            float s = 0.0f;
            for (int64_t i = threadIdx.x; i < p.L; i += THREADS) s += load_as<float>(p.in, p.dtype, ib + i * p.in_ax_stride);
            a = block_reduce(s, false, sh) / fL;
            float sq = 0.0f;
            for (int64_t i = threadIdx.x; i < p.L; i += THREADS) {
                float d = load_as<float>(p.in, p.dtype, ib + i * p.in_ax_stride) - a;
                sq += d * d;
            }
            const float var = block_reduce(sq, false, sh) / fL;
            b = (p.mode == M_LN_ONNX) ? 1.0f / sqrtf(var + p.eps) : 1.0f / (sqrtf(var) + p.eps);
        }
        for (int64_t i = threadIdx.x; i < p.L; i += THREADS) {
            float v = load_as<float>(p.in, p.dtype, ib + i * p.in_ax_stride);
            float r;
            if (p.mode == M_SOFTMAX) r = expf(v - a) * b;
            else if (p.mode == M_RMS) r = v * b;
            else {
                r = (v - a) * b;
                if (p.gamma) r = r * load_as<float>(p.gamma, p.g_dtype, i * p.g_stride);
                if (p.beta) r = r + load_as<float>(p.beta, p.b_dtype, i * p.b_stride);
            }
            store_from(p.out, p.out_dtype, ob + i * p.out_ax_stride, r);
        }
        __syncthreads();  // all reads of this row done before a possible in-place next row
    }
}

// ------------------------------------------------------------- host side --

int blocks_per_sm(const void* fn) {
    static std::mutex mu;
    static std::unordered_map<const void*, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(fn);
    if (it != cache.end()) return it->second;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, THREADS, 0) != cudaSuccess || nb <= 0) nb = 1;
    cache[fn] = nb;
    return nb;
}

template <typename T, int CH, int MODE>
int launch_warp(const NormParams& p, cudaStream_t s) {
    // Persistent: resident CTAs only, each warp walking rows.  Launching one
    // CTA per 8 rows (the block scheduler balancing SMs, which wins for the
    // streaming kernels) measured slower here: config 4 at 5354 GB/s with one
    // row per warp, 6043 with 4 and 6138 with 16, against 6185 persistent; a
    // warp's row ends in a reduction whose latency the next row hides.
    const void* fn = (const void*)rownorm_warp_kernel<T, CH, MODE>;
    int64_t want = (p.nrows + (THREADS / 32) - 1) / (THREADS / 32);
    int64_t cap = (int64_t)sm_count() * blocks_per_sm(fn);
    int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
    (void)launch_pdl(rownorm_warp_kernel<T, CH, MODE>, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "row-norm launch");
}

template <typename T, int MODE>
int launch_ch(int ch, const NormParams& p, cudaStream_t s) {
    switch (ch) {
    case 1: return launch_warp<T, 1, MODE>(p, s);
    case 2: return launch_warp<T, 2, MODE>(p, s);
    case 4: return launch_warp<T, 4, MODE>(p, s);
    default: return launch_warp<T, 8, MODE>(p, s);
    }
}

// Kernel MODE = the row op, + 4 when gamma/beta take the per-element path.
template <typename T>
int launch_mode(int mode, int ch, const NormParams& p, cudaStream_t s) {
    const bool gbv = p.gb_vec != 0;
    switch (mode) {
    case M_SOFTMAX: return launch_ch<T, M_SOFTMAX>(ch, p, s);
    case M_LN_ONNX: return gbv ? launch_ch<T, M_LN_ONNX>(ch, p, s) : launch_ch<T, M_LN_ONNX | 4>(ch, p, s);
    case M_LN_TADMA: return gbv ? launch_ch<T, M_LN_TADMA>(ch, p, s) : launch_ch<T, M_LN_TADMA | 4>(ch, p, s);
    default: return launch_ch<T, M_RMS>(ch, p, s);
    }
}

int run_rownorm(int mode, const tadma_tensor* in, int32_t axis, const tadma_tensor* gamma, const tadma_tensor* beta,
                double eps, const tadma_tensor* out, cudaStream_t s) {
    std::string err = check_tensor(in, "in");
    if (err.empty()) err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (in->rank < 1) return fail(TADMA_ERR_INVALID, "rank must be >= 1");
    if (out->rank != in->rank) return fail(TADMA_ERR_INVALID, "out rank differs from in rank");
    for (int d = 0; d < in->rank; d++)
        if (out->dims[d] != in->dims[d]) return fail(TADMA_ERR_INVALID, "out dims differ from in dims");
    if (!dtype_is_float(in->dtype) || !dtype_is_float(out->dtype)) return fail(TADMA_ERR_INVALID, "float dtypes only");
    const int ax = axis < 0 ? axis + in->rank : axis;
    if (ax < 0 || ax >= in->rank) return fail(TADMA_ERR_INVALID, "axis out of range");
    const int64_t L = in->dims[ax];
    NormParams p{};
    p.in = (const char*)in->data;
    p.out = (char*)out->data;
    p.dtype = in->dtype;
    p.out_dtype = out->dtype;
    p.mode = mode;
    p.eps = (float)eps;
    p.L = L;
    p.in_ax_stride = in->strides[ax];
    p.out_ax_stride = out->strides[ax];
    for (int k = 0; k < 2; k++) {
        const tadma_tensor* t = k == 0 ? gamma : beta;
        if (!t || !t->data) continue;
        err = check_tensor(t, k == 0 ? "gamma" : "beta");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (t->rank != 1 || t->dims[0] != L) return fail(TADMA_ERR_INVALID, "gamma/beta must be 1-D of the normalised length");
        if (k == 0) {
            p.gamma = (const char*)t->data;
            p.g_dtype = t->dtype;
            p.g_stride = t->strides[0];
        } else {
            p.beta = (const char*)t->data;
            p.b_dtype = t->dtype;
            p.b_stride = t->strides[0];
        }
    }
    if (numel(in) == 0) return TADMA_OK;

    int64_t kd[TADMA_MAX_RANK], ks[2][TADMA_MAX_RANK];
    int kr = 0;
    for (int d = 0; d < in->rank; d++) {
        if (d == ax) continue;
        kd[kr] = in->dims[d];
        ks[0][kr] = in->strides[d];
        ks[1][kr] = out->strides[d];
        kr++;
    }
    Folded f = fold(kr, kd, ks, 2);
    p.nrows = 1;
    for (int d = 0; d < f.rank; d++) p.nrows *= f.dims[d];

    const int dt = in->dtype;
    const int es = dtype_size(dt);
    const int N = 16 / es;
    const bool fast_dt = (dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16) && out->dtype == dt;
    const int64_t cap = 32LL * N * 8;
    if (fast_dt && f.rank == 1 && p.in_ax_stride == 1 && p.out_ax_stride == 1 && L % N == 0 && L <= cap &&
        (uintptr_t)in->data % 16 == 0 && (uintptr_t)out->data % 16 == 0 &&
        (f.strides[0][0] * es) % 16 == 0 && (f.strides[1][0] * es) % 16 == 0) {
        p.in_row_stride = f.strides[0][0];
        p.out_row_stride = f.strides[1][0];
        p.gb_vec = 1;
        for (int k = 0; k < 2; k++) {
            const char* ptr = k == 0 ? p.gamma : p.beta;
            if (!ptr) continue;
            int gdt = k == 0 ? p.g_dtype : p.b_dtype;
            int64_t gs = k == 0 ? p.g_stride : p.b_stride;
            if (gdt != dt || gs != 1 || (uintptr_t)ptr % 16) p.gb_vec = 0;
        }
        const int64_t per = 32LL * N;
        int ch = (int)((L + per - 1) / per);
        ch = ch <= 1 ? 1 : ch <= 2 ? 2 : ch <= 4 ? 4 : 8;
        switch (dt) {
        case TADMA_F32: return launch_mode<float>(mode, ch, p, s);
        case TADMA_F16: return launch_mode<__half>(mode, ch, p, s);
        default: return launch_mode<__nv_bfloat16>(mode, ch, p, s);
        }
    }
    p.krank = f.rank;
    for (int d = 0; d < f.rank; d++) {
        p.kdm[d] = DivMod((uint64_t)f.dims[d]);
        p.kin[d] = f.strides[0][d];
        p.kout[d] = f.strides[1][d];
    }
    int64_t cap_blocks = (int64_t)sm_count() * blocks_per_sm((const void*)rownorm_block_kernel);
    int grid = (int)(p.nrows < cap_blocks ? p.nrows : cap_blocks);
    (void)launch_pdl(rownorm_block_kernel, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "row-norm launch");
}

}  // namespace

}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_softmax(const tadma_tensor* in, int32_t axis, const tadma_tensor* out, void* stream) {
    return run_rownorm(M_SOFTMAX, in, axis, nullptr, nullptr, 0.0, out, (cudaStream_t)stream);
}

extern "C" int tadma_b200_layer_norm(const tadma_tensor* in, int32_t axis, const tadma_tensor* gamma,
                                     const tadma_tensor* beta, double eps, int32_t mode, const tadma_tensor* out,
                                     void* stream) {
    if (mode != TADMA_LN_ONNX && mode != TADMA_LN_TADMA) return fail(TADMA_ERR_INVALID, "unknown layer-norm mode");
    if (in) {
        const int ax = axis < 0 ? axis + in->rank : axis;
        if (ax != in->rank - 1) return fail(TADMA_ERR_UNSUPPORTED, "layer_norm: only the last axis");
    }
    return run_rownorm(mode == TADMA_LN_ONNX ? M_LN_ONNX : M_LN_TADMA, in, axis, gamma, beta, eps, out,
                       (cudaStream_t)stream);
}

extern "C" int tadma_b200_rms_norm(const tadma_tensor* in, int32_t axis, double eps, const tadma_tensor* out,
                                   void* stream) {
    return run_rownorm(M_RMS, in, axis, nullptr, nullptr, eps, out, (cudaStream_t)stream);
}
