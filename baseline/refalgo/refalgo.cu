// refalgo.cu - "reference algorithm, restated": TADMA's own GPU kernels as
// they would run on this B200, for timing next to tadma_b200.  NOT the product
// and NOT the oracle; bench.py (its reference_gpu_restated object) launches
// it, and tests/test_reference_order_gpu.py checks the oracle's
// reference-order reduction against its ReduceKernel.
//
// The reference (OgnianM/TADMA) cannot be compiled here (C++23 / clang >= 19),
// so its three kernels are restated with their exact launch geometry and
// per-thread algorithm, and composed the way its API composes them:
// * executor  - CUDAHIPExecutorKernel (include/tadma/Node.hpp:25-48): 512
//   threads, one element per thread, 32-bit index, MapToShape div/mod by
//   compile-time dims (Utils.hpp:9-17), guard only when Product % 512 != 0;
// * gather    - EltwiseVariadicNDKernel (kernels/EltwiseVariadicND.hpp:6-27):
//   256 threads, one element per thread, no bounds guard;
// * reduce    - ReduceKernel<Threads> (kernels/Reduce.hpp:10-69): one block
//   per output over the transpose<D,0> view, Threads = min(1024,
//   floor_pow2(Dim)), strided per-thread fold, shared-memory tree with a
//   __syncthreads per level, accumulation in decltype(a + b) (fp16 in fp16).
// Compositions: config 2 = x*0.5f (float node) -> + bias (float node) ->
// gelu<true> (double math, Operations.hpp:181); softmax = exp<true> -> sum
// reduce -> in-place divide (Operations.hpp:190-193); LayerNorm = mean reduce
// -> squared-difference reduce with sqrt post -> normalise node
// (Operations.hpp:195-220); gather + pos = gather node -> add node.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace {

// ---------------------------------------------------------------- executor --
template <int64_t D0, int64_t D1, typename F>
__global__ void exec2_kernel(F f) {
    constexpr int64_t Product = D0 * D1;
    unsigned index = blockIdx.x * blockDim.x + threadIdx.x;  // 32-bit, as Node.hpp:28
    if constexpr (Product % 512 != 0) {
        if (index >= Product) return;
    }
    int64_t idx = index;
    const int64_t i1 = idx % D1;  // MapToShape peels the last dim first
    idx /= D1;
    const int64_t i0 = idx % D0;
    f(i0, i1);
}

template <int64_t D0, int64_t D1, typename F>
void exec2(F f, cudaStream_t s) {
    constexpr int64_t Product = D0 * D1;
    exec2_kernel<D0, D1><<<(unsigned)((Product + 511) / 512), 512, 0, s>>>(f);
}

__device__ double tanh_ref(double x) {  // Operations.hpp:160-164
    double en = exp(-x), ep = exp(x);
    return (ep - en) / (ep + en);
}

// ----------------------------------------------------------------- reduce --
// One block per output; element i of output g sits at base(g) + i * rstride.
// The group index walks the kept dims of the transpose<D,0> view in MapToShape
// order: gi = g % inner is the fastest kept dim (input stride inner_stride,
// output stride out_is), go = g / inner the other (outer_stride, out_os).
template <int Threads, typename T, typename Acc, int OP>  // OP 0 sum, 1 max, 2 mean, 3 sq-diff-sum
__global__ void reduce_kernel(const T* x, Acc* out, int64_t R, int64_t rstride, int64_t inner, int64_t inner_stride,
                              int64_t outer_stride, int64_t out_is, int64_t out_os, const Acc* center, int post_sqrt) {
    __shared__ Acc shared[Threads];
    const unsigned tid = threadIdx.x;
    const unsigned g = blockIdx.x;
    const int64_t gi = g % inner, go = g / inner;
    const T* base = x + go * outer_stride + gi * inner_stride;
    auto pre = [&](T v) -> Acc {
        if constexpr (OP == 3) {
            Acc d = (Acc)v - center[g];
            return d * d;
        } else {
            return (Acc)v;
        }
    };
    if (tid < R) {
        Acc value = pre(base[(int64_t)tid * rstride]);
        for (int64_t idx = tid + Threads; idx < R; idx += Threads) {
            Acc v = pre(base[idx * rstride]);
            value = (OP == 1) ? (value < v ? v : value) : value + v;
        }
        shared[tid] = value;
    }
    __syncthreads();
    for (int i = Threads >> 1; i > 0; i >>= 1) {
        if (tid < i && (int64_t)(tid + i) < R) {
            Acc a = shared[tid], b = shared[tid + i];
            shared[tid] = (OP == 1) ? (a < b ? b : a) : a + b;
        }
        __syncthreads();
    }
    if (tid == 0) {
        Acc r = shared[0];
        if (OP == 2) r = r / (Acc)(float)R;
        if (post_sqrt) r = (Acc)sqrtf((float)r / (float)R);
        out[gi * out_is + go * out_os] = r;
    }
}

int threads_for(int64_t R) {
    int t = 1;
    while ((int64_t)t * 2 <= R && t < 1024) t *= 2;
    return t;
}

template <typename T, typename Acc, int OP>
void reduce(const T* x, Acc* out, int64_t nout, int64_t R, int64_t rstride, int64_t inner, int64_t inner_stride,
            int64_t outer_stride, int64_t out_is, int64_t out_os, const Acc* center, int post_sqrt, cudaStream_t s) {
#define TADMA_REF_RED(TH)                                                                                    \
    reduce_kernel<TH, T, Acc, OP><<<(unsigned)nout, TH, 0, s>>>(x, out, R, rstride, inner, inner_stride, \
                                                                 outer_stride, out_is, out_os, center, post_sqrt)
    switch (threads_for(R)) {
    case 1024: TADMA_REF_RED(1024); break;
    case 512: TADMA_REF_RED(512); break;
    case 256: TADMA_REF_RED(256); break;
    default: TADMA_REF_RED(128); break;
    }
#undef TADMA_REF_RED
}

// ----------------------------------------------------------------- gather --
template <int64_t B, int64_t S, int64_t D>
__global__ void gather_kernel(const __half* table, const int64_t* ids, __half* out) {
    const unsigned idx = blockIdx.x * blockDim.x + threadIdx.x;  // no guard, 32-bit
    int64_t e = idx;
    const int64_t d = e % D;
    e /= D;
    const int64_t s = e % S;
    const int64_t b = e / S;
    const int64_t id = ids[b * S + s];
    out[(b * S + s) * D + d] = table[id * D + d];
}

}  // namespace

extern "C" {

// config 1: t = A + b (float node), exp<true>(t) in place, sum<-1>(t) through
// ReduceKernel<128>.  A [64, 128], b [128] fp32 -> y [64].
int ref_cfg1(const void* A, const void* b, void* t, void* y, void* stream) {
    constexpr int64_t R = 64, C = 128;
    cudaStream_t s = (cudaStream_t)stream;
    const float* ap = (const float*)A;
    const float* bp = (const float*)b;
    float* tp = (float*)t;
    exec2<R, C>([=] __device__(int64_t i, int64_t j) { tp[i * C + j] = ap[i * C + j] + bp[j]; }, s);
    exec2<R, C>([=] __device__(int64_t i, int64_t j) { tp[i * C + j] = expf(tp[i * C + j]); }, s);
    reduce<float, float, 0>(tp, (float*)y, R, C, 1, R, C, 0, 1, 0, nullptr, 0, s);
    return (int)cudaGetLastError();
}

// config 2: t1 = x * 0.5f; t2 = t1 + bias; gelu<true>(t2).  x, bias bf16; t1, t2 fp32 [8192, 8192].
int ref_cfg2(const void* x, const void* bias, void* t1, void* t2, void* stream) {
    constexpr int64_t R = 8192, C = 8192;
    cudaStream_t s = (cudaStream_t)stream;
    const __nv_bfloat16* xp = (const __nv_bfloat16*)x;
    const __nv_bfloat16* bp = (const __nv_bfloat16*)bias;
    float* a = (float*)t1;
    float* o = (float*)t2;
    exec2<R, C>([=] __device__(int64_t i, int64_t j) { a[i * C + j] = __bfloat162float(xp[i * C + j]) * 0.5f; }, s);
    exec2<R, C>([=] __device__(int64_t i, int64_t j) { o[i * C + j] = a[i * C + j] + __bfloat162float(bp[j]); }, s);
    exec2<R, C>([=] __device__(int64_t i, int64_t j) {
        double xv = o[i * C + j];
        o[i * C + j] = (float)(0.5 * xv * (1 + tanh_ref(0.7978845608 * (xv + 0.044715 * xv * xv * xv))));
    }, s);
    return (int)cudaGetLastError();
}

// config 3: sum and max over axis 2, mean over axis 1 of X[32, 4096, 4096] fp32.
int ref_cfg3(const void* x, void* sum_out, void* max_out, void* mean_out, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    const float* xp = (const float*)x;
    // axis 2: transpose<2,0> view [4096 (i), 4096 (r), 32 (b)]; group g -> (r, b) = (g / 32, g % 32)
    reduce<float, float, 0>(xp, (float*)sum_out, 32 * 4096, 4096, 1, 32, 4096LL * 4096, 4096, 4096, 1, nullptr, 0, s);
    reduce<float, float, 1>(xp, (float*)max_out, 32 * 4096, 4096, 1, 32, 4096LL * 4096, 4096, 4096, 1, nullptr, 0, s);
    // axis 1: transpose<1,0> view [4096 (i), 32 (b), 4096 (j)]; group g -> (b, j); lanes read 16 KB apart
    reduce<float, float, 2>(xp, (float*)mean_out, 32 * 4096, 4096, 4096, 4096, 1, 4096LL * 4096, 1, 4096, nullptr, 0, s);
    return (int)cudaGetLastError();
}

// config 4 softmax: e = exp<true>(x); sum<-1> (fp16 accumulation); e /= sum.  x [32*16*2048, 2048] fp16, in place.
int ref_cfg4_softmax(void* x, void* sums, int64_t rows, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    __half* xp = (__half*)x;
    __half* sp = (__half*)sums;
    constexpr int64_t L = 2048;
    constexpr int64_t ROWS = 32LL * 16 * 2048;
    if (rows != ROWS) return -1;
    exec2<ROWS, L>([=] __device__(int64_t i, int64_t j) { xp[i * L + j] = __float2half(expf(__half2float(xp[i * L + j]))); }, s);
    reduce<__half, __half, 0>(xp, sp, ROWS, L, 1, ROWS, L, 0, 1, 0, nullptr, 0, s);
    exec2<ROWS, L>([=] __device__(int64_t i, int64_t j) { xp[i * L + j] = __hdiv(xp[i * L + j], sp[i]); }, s);
    return (int)cudaGetLastError();
}

// config 4 LayerNorm (reference formula): mean, std = sqrt(sum((x-mean)^2)/n),
// y = (x - mean) / (std + eps) * gamma + beta.  x [64*2048, 1024] fp16 -> y.
int ref_cfg4_ln(const void* x, const void* gamma, const void* beta, void* mean, void* stdv, void* y, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    constexpr int64_t ROWS = 64LL * 2048, L = 1024;
    const __half* xp = (const __half*)x;
    __half* mp = (__half*)mean;
    __half* sp = (__half*)stdv;
    const __half* gp = (const __half*)gamma;
    const __half* bp = (const __half*)beta;
    __half* yp = (__half*)y;
    reduce<__half, __half, 2>(xp, mp, ROWS, L, 1, ROWS, L, 0, 1, 0, nullptr, 0, s);
    reduce<__half, __half, 3>(xp, sp, ROWS, L, 1, ROWS, L, 0, 1, 0, mp, 1, s);
    exec2<ROWS, L>([=] __device__(int64_t i, int64_t j) {
        float v = (__half2float(xp[i * L + j]) - __half2float(mp[i])) / (__half2float(sp[i]) + 1e-5f);
        yp[i * L + j] = __float2half(v * __half2float(gp[j]) + __half2float(bp[j]));
    }, s);
    return (int)cudaGetLastError();
}

// config 5 at batch 64 (the reference's 32-bit index cannot cover batch 2048):
// g = gather(table, ids) (fp16) then out = g + pos (float, as the C++ types promote).
int ref_cfg5_b64(const void* table, const void* ids, const void* pos, void* g, void* out, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
    constexpr int64_t B = 64, S = 4096, D = 4096;
    const __nv_bfloat16* pp = (const __nv_bfloat16*)pos;
    __half* gp = (__half*)g;
    float* op = (float*)out;
    gather_kernel<B, S, D><<<(unsigned)(B * S * D / 256), 256, 0, s>>>((const __half*)table, (const int64_t*)ids, gp);
    exec2<B * S, D>([=] __device__(int64_t r, int64_t d) {
        op[r * D + d] = __half2float(gp[r * D + d]) + __bfloat162float(pp[(r % S) * D + d]);
    }, s);
    return (int)cudaGetLastError();
}

// A row reduction through ReduceKernel alone, for the parity test of the
// oracle's reference-order mode: x [rows, R] contiguous, fp32 (dtype 0) or
// fp16 (dtype 1, accumulated in fp16); op 0 sum, 1 max, 2 mean.
int ref_reduce_rows(const void* x, int dtype, void* out, int64_t rows, int64_t R, int op, void* stream) {
    cudaStream_t s = (cudaStream_t)stream;
#define TADMA_REF_ROWS(T, OPC) reduce<T, T, OPC>((const T*)x, (T*)out, rows, R, 1, rows, R, 0, 1, 0, nullptr, 0, s)
    if (dtype == 0) {
        if (op == 0) TADMA_REF_ROWS(float, 0);
        else if (op == 1) TADMA_REF_ROWS(float, 1);
        else TADMA_REF_ROWS(float, 2);
    } else {
        if (op == 0) TADMA_REF_ROWS(__half, 0);
        else if (op == 1) TADMA_REF_ROWS(__half, 1);
        else TADMA_REF_ROWS(__half, 2);
    }
#undef TADMA_REF_ROWS
    return (int)cudaGetLastError();
}

}  // extern "C"
