// chain_reduce.cu - tadma_b200_reduce_chain's kernel: a reduction whose
// elements are a fused chain, evaluated on the fly.
#include "eltwise_impl.cuh"

namespace tadma_b200 {
namespace {

// ------------------------------------------------------ chain reduction --
//
// tadma_b200_reduce_chain: a reduction whose elements are a fused chain of
// up to 6 broadcast operands, evaluated on the fly.  One warp per output
// element (the kept dims, folded); its lanes walk the reduced axis.  With the
// axis contiguous (stride 1) or broadcast (stride 0) in every operand and
// fp32 compute, lanes take 8 elements per step with 16-byte loads (the
// eltwise vector loader) and run the chain on the 8 at once; otherwise one
// element per lane step.  Lanes fold their elements in increasing index
// order and combine in a fixed butterfly, as the reduction kernels do.

// Raw 16-byte words of one 8-element vector (fp32: 2 words, fp16 / bf16: 1),
// converted to the compute type at use.
struct RawV {
    uint4 a, b;
};
__device__ __forceinline__ void load_raw_vec(const Operand& o, int64_t off, RawV& r) {
    const char* p = o.base + off * dtype_size(o.dtype);
    r.a = ld_stream_v4(p);
    if (o.dtype == TADMA_F32) r.b = ld_stream_v4(p + 16);
}
template <typename C>
__device__ __forceinline__ void cvt_raw_vec(int dt, const RawV& r, C (&v)[V]) {
    if (dt == TADMA_F32) {
        const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = from_f<C>(__uint_as_float(w[j]));
    } else {
        float f[8];
        unpack8(r.a, dt, f);
#pragma unroll
        for (int j = 0; j < V; j++) v[j] = from_f<C>(f[j]);
    }
}



template <typename C, int K, bool VEC, int NIN>
__global__ void __launch_bounds__(THREADS, !VEC ? 2 : NIN == 1 ? 3 : NIN <= 4 ? 2 : 1) chain_reduce_kernel(const __grid_constant__ ChainReduceParams p) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    for (int64_t row = gw; row < p.nrows; row += nw) {
        int64_t base[TADMA_MAX_INPUTS] = {};
        int64_t ooff = 0;
        {
            uint64_t e = (uint64_t)row;
            for (int d = p.krank - 1; d >= 0; d--) {
                uint64_t q, r;
                if (d > 0) {
                    p.kdm[d].divmod(e, q, r);
                } else {
                    r = e;
                    q = 0;
                }
                ooff += (int64_t)r * p.kout[d];
#pragma unroll
                for (int k = 0; k < TADMA_MAX_INPUTS; k++) base[k] += (int64_t)r * p.kin[k][d];
                e = q;
            }
        }
        State<C> s = init_state<K, C>();
        int64_t done = 0;
        if constexpr (VEC) {
            // An operand broadcast along the axis is one value per output,
            // loaded once.  The others are double-buffered as raw 16-byte
            // words: the next vector step's loads are in flight while this
            // step converts, runs the chain and folds.
            const int64_t nv = p.R / V;
            C bc[NIN];
#pragma unroll
            for (int k = 0; k < NIN; k++)
                bc[k] = p.ax[k] == 0 ? load_as<C>(p.chain.in[k].base, p.chain.in[k].dtype, base[k]) : C(0);
            RawV cur[NIN], nxt[NIN];
            int64_t v = lane;
            if (v < nv) {
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    if (p.ax[k] != 0) load_raw_vec(p.chain.in[k], base[k] + v * V, cur[k]);
            }
            for (; v < nv; v += 32) {
                if (v + 32 < nv) {
#pragma unroll
                    for (int k = 0; k < NIN; k++)
                        if (p.ax[k] != 0) load_raw_vec(p.chain.in[k], base[k] + (v + 32) * V, nxt[k]);
                }
                C val[NIN][V];
#pragma unroll
                for (int k = 0; k < NIN; k++) {
                    if (p.ax[k] == 0) {
#pragma unroll
                        for (int j = 0; j < V; j++) val[k][j] = bc[k];
                    } else {
                        cvt_raw_vec<C>(p.chain.in[k].dtype, cur[k], val[k]);
                    }
                }
                C acc[V];
#pragma unroll
                for (int j = 0; j < V; j++) acc[j] = val[0][j];
                run_chain<C, NIN, V, false>(p.chain, acc, val);
#pragma unroll
                for (int j = 0; j < V; j++) update<K, C>(s, p.square ? sq(acc[j]) : acc[j], v * V + j);
#pragma unroll
                for (int k = 0; k < NIN; k++) cur[k] = nxt[k];
            }
            done = nv * V;
        }
        for (int64_t r = done + lane; r < p.R; r += 32) {
            C val[TADMA_MAX_INPUTS][1];
#pragma unroll
            for (int k = 0; k < TADMA_MAX_INPUTS; k++)
                if (k < p.n_ins) val[k][0] = load_as<C>(p.chain.in[k].base, p.chain.in[k].dtype, base[k] + r * p.ax[k]);
            C acc[1] = {p.n_ins > 0 ? val[0][0] : C(0)};
            run_chain<C, TADMA_MAX_INPUTS, 1, false>(p.chain, acc, val);
            update<K, C>(s, p.square ? sq(acc[0]) : acc[0], r);
        }
        s = warp_combine<K, C>(s);
        if (lane == 0) {
            if constexpr (K == K_ARGMAX || K == K_ARGMIN) {
                store_from(p.out, p.out_dtype, ooff, (int64_t)(s.i < 0 ? 0 : s.i));
            } else {
                C v = s.v;
                if constexpr (std::is_floating_point<C>::value) {
                    if (p.post == POST_MEAN) v = v / (C)p.R;
                    else if (p.post == POST_RMS) v = sqrt(v / (C)p.R);
                } else {
                    if (p.post == POST_MEAN) v = v / p.R;
                }
                if (p.pc.n) v = apply_post<C>(p.pc, v);
                store_from(p.out, p.out_dtype, ooff, v);
            }
        }
    }
}

// Typed vector path (fp32 compute): every operand either streams along the
// reduced axis (stride 1, one dtype T for all of them, 16-byte aligned rows)
// or is broadcast along it (one value per output, loaded once).  Lanes take
// 16-byte vectors of T (4 fp32 or 8 16-bit values): UNR of them per streamed
// operand are loaded before any is used (64 bytes per operand in flight per
// lane with one or two operands), then a rolled loop runs the pre-decoded
// program on G vectors at a time (W = G x N = 8 values per step with up to
// four operands) and shifts the next G down.  Values fold in increasing
// index order.
template <typename T, int NIN>
struct TypedShape {
    static constexpr int N = 16 / (int)sizeof(T);
    static constexpr int UNR = NIN <= 2 ? 4 : NIN <= 4 ? 2 : (sizeof(T) == 4 ? 2 : 1);
    static constexpr int G = sizeof(T) == 4 && NIN <= 4 ? 2 : 1;
    static constexpr int W = G * N;
};

template <typename T>
__device__ __forceinline__ void cvt_typed(uint4 r, float* f) {
    if constexpr (sizeof(T) == 4) {
        f[0] = __uint_as_float(r.x);
        f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z);
        f[3] = __uint_as_float(r.w);
    } else {
        unpack8(r, std::is_same<T, __half>::value ? TADMA_F16 : TADMA_BF16, f);
    }
}

template <typename T, int K, int NIN>
__global__ void __launch_bounds__(THREADS, NIN <= 2 ? 3 : 2) chain_reduce_typed_kernel(const __grid_constant__ ChainReduceParams p) {
    pdl_begin();
    using S = TypedShape<T, NIN>;
    constexpr int N = S::N, UNR = S::UNR, G = S::G, W = S::W;
    const int lane = threadIdx.x & 31;
    extern __shared__ uint4 cr_ring[];
    uint4* ring = cr_ring + (threadIdx.x >> 5) * (2 * NIN * UNR * 32);  // 2 stages x NIN x UNR x 32 lanes
    const int64_t gw = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
    const int64_t nw = ((int64_t)gridDim.x * THREADS) >> 5;
    for (int64_t row = gw; row < p.nrows; row += nw) {
        int64_t base[NIN];
        int64_t ooff = 0;
#pragma unroll
        for (int k = 0; k < NIN; k++) base[k] = 0;
        {
            uint64_t e = (uint64_t)row;
            for (int d = p.krank - 1; d >= 0; d--) {
                uint64_t q, r;
                if (d > 0) {
                    p.kdm[d].divmod(e, q, r);
                } else {
                    r = e;
                    q = 0;
                }
                ooff += (int64_t)r * p.kout[d];
#pragma unroll
                for (int k = 0; k < NIN; k++) base[k] += (int64_t)r * p.kin[k][d];
                e = q;
            }
        }
        float bc[NIN];
#pragma unroll
        for (int k = 0; k < NIN; k++)
            bc[k] = p.ax[k] == 0 ? load_as<float>(p.chain.in[k].base, p.chain.in[k].dtype, base[k]) : 0.0f;
        State<float> s = init_state<K, float>();
        const int64_t nv = p.R / N;
        // Vectors i0, i0 + 32, ..., i0 + 32 (UNR - 1) of every streamed
        // operand go into this lane's slots of the warp's two-stage ring
        // with cp.async; the next group's copies are issued before the
        // current group is computed.  Each lane reads back only what it
        // copied, so its own wait_group orders copy and use.  Slots past the
        // row's last vector keep stale words: computed, never folded.
        auto issue = [&](int64_t g0, int st) {
#pragma unroll
            for (int u = 0; u < UNR; u++) {
#pragma unroll
                for (int k = 0; k < NIN; k++) {
                    if (p.ax[k] != 0 && g0 + 32 * u < nv)
                        cp_async16(ring + ((st * NIN + k) * UNR + u) * 32 + lane,
                                   reinterpret_cast<const T*>(p.chain.in[k].base) + base[k] + (g0 + 32 * u) * N);
                }
            }
            cp_async_commit();
        };
        int st = 0;
        issue(lane, 0);
        for (int64_t i0 = lane; i0 < nv; i0 += 32 * UNR, st ^= 1) {
            issue(i0 + 32 * UNR, st ^ 1);
            cp_async_wait<1>();
#pragma unroll 1
            for (int h = 0; h < UNR / G; h++) {
                float val[NIN][W];
#pragma unroll
                for (int k = 0; k < NIN; k++) {
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        if (p.ax[k] == 0) {
#pragma unroll
                            for (int j = 0; j < N; j++) val[k][g * N + j] = bc[k];
                        } else {
                            cvt_typed<T>(ring[((st * NIN + k) * UNR + h * G + g) * 32 + lane], &val[k][g * N]);
                        }
                    }
                }
                float acc[W];
#pragma unroll
                for (int j = 0; j < W; j++) acc[j] = val[0][j];
                run_fprog<NIN, W, false>(p.chain.fp, acc, val);
#pragma unroll
                for (int g = 0; g < G; g++) {
                    const int64_t vg = i0 + 32 * (h * G + g);
                    if (vg < nv) {
#pragma unroll
                        for (int j = 0; j < N; j++) {
                            const float a = acc[g * N + j];
                            update<K, float>(s, p.square ? sq(a) : a, vg * N + j);
                        }
                    }
                }
            }
        }
        cp_async_wait<0>();  // the last (empty) group, before the ring's reuse
        for (int64_t r = nv * N + lane; r < p.R; r += 32) {
            float val[NIN][1];
#pragma unroll
            for (int k = 0; k < NIN; k++) val[k][0] = load_as<float>(p.chain.in[k].base, p.chain.in[k].dtype, base[k] + r * p.ax[k]);
            float acc[1] = {val[0][0]};
            run_fprog<NIN, 1, false>(p.chain.fp, acc, val);
            update<K, float>(s, p.square ? sq(acc[0]) : acc[0], r);
        }
        s = warp_combine<K, float>(s);
        if (lane == 0) {
            if constexpr (K == K_ARGMAX || K == K_ARGMIN) {
                store_from(p.out, p.out_dtype, ooff, (int64_t)(s.i < 0 ? 0 : s.i));
            } else {
                float v = s.v;
                if (p.post == POST_MEAN) v = v / (float)p.R;
                else if (p.post == POST_RMS) v = sqrtf(v / (float)p.R);
                if (p.pc.n) v = apply_post<float>(p.pc, v);
                store_from(p.out, p.out_dtype, ooff, v);
            }
        }
    }
}

template <typename T, int K, int NIN>
int launch_typed_k(const ChainReduceParams& p, cudaStream_t s) {
    using S = TypedShape<T, NIN>;
    const void* fn = (const void*)chain_reduce_typed_kernel<T, K, NIN>;
    const size_t smem = (size_t)(THREADS / 32) * 2 * NIN * S::UNR * 32 * 16;
    // the shared-memory attribute and the occupancy, once per device (the
    // attribute belongs to the device's context)
    static thread_local int occ[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_reduce_chain cudaGetDevice");
    int& per_sm = occ[dev & 63];
    if (per_sm <= 0) {
        if (smem > 48 * 1024) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, THREADS, smem);
        if (e != cudaSuccess) {
            per_sm = 0;
            return cuda_fail(e, "tadma_b200_reduce_chain kernel setup");
        }
    }
    const int64_t want = (p.nrows + (THREADS / 32) - 1) / (THREADS / 32);
    const int64_t cap = (int64_t)sm_count() * (per_sm > 0 ? per_sm : 1);
    const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
    e = launch_pdl(chain_reduce_typed_kernel<T, K, NIN>, dim3(grid), dim3(THREADS), smem, s, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_reduce_chain launch");
}

template <typename T, int NIN>
int launch_typed_n(int kind, const ChainReduceParams& p, cudaStream_t s) {
    switch (kind) {
    case K_SUM: return launch_typed_k<T, K_SUM, NIN>(p, s);
    case K_MAX: return launch_typed_k<T, K_MAX, NIN>(p, s);
    case K_MIN: return launch_typed_k<T, K_MIN, NIN>(p, s);
    case K_ARGMAX: return launch_typed_k<T, K_ARGMAX, NIN>(p, s);
    default: return launch_typed_k<T, K_ARGMIN, NIN>(p, s);
    }
}

template <typename T>
int launch_typed_t(int kind, const ChainReduceParams& p, cudaStream_t s) {
    switch (p.n_ins) {
    case 1: return launch_typed_n<T, 1>(kind, p, s);
    case 2: return launch_typed_n<T, 2>(kind, p, s);
    case 3: return launch_typed_n<T, 3>(kind, p, s);
    case 4: return launch_typed_n<T, 4>(kind, p, s);
    case 5: return launch_typed_n<T, 5>(kind, p, s);
    default: return launch_typed_n<T, 6>(kind, p, s);
    }
}

template <typename C, int K, bool VEC, int NIN>
int launch_chain_reduce_k(const ChainReduceParams& p, cudaStream_t s) {
    const void* fn = (const void*)chain_reduce_kernel<C, K, VEC, NIN>;
    const int64_t want = (p.nrows + (THREADS / 32) - 1) / (THREADS / 32);
    const int64_t cap = (int64_t)sm_count() * blocks_per_sm(fn);
    const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
    cudaError_t e = launch_pdl(chain_reduce_kernel<C, K, VEC, NIN>, dim3(grid), dim3(THREADS), 0, s, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_reduce_chain launch");
}

// The scalar path takes the operand count at run time (NIN = 4 arrays); the
// vector path is instantiated per operand count to keep its registers.
template <typename C, bool VEC, int NIN>
int launch_chain_reduce_n(int kind, const ChainReduceParams& p, cudaStream_t s) {
    switch (kind) {
    case K_SUM: return launch_chain_reduce_k<C, K_SUM, VEC, NIN>(p, s);
    case K_MAX: return launch_chain_reduce_k<C, K_MAX, VEC, NIN>(p, s);
    case K_MIN: return launch_chain_reduce_k<C, K_MIN, VEC, NIN>(p, s);
    case K_ARGMAX: return launch_chain_reduce_k<C, K_ARGMAX, VEC, NIN>(p, s);
    default: return launch_chain_reduce_k<C, K_ARGMIN, VEC, NIN>(p, s);
    }
}

template <typename C, bool VEC>
int launch_chain_reduce(int kind, const ChainReduceParams& p, cudaStream_t s) {
    if constexpr (!VEC) {
        return launch_chain_reduce_n<C, false, TADMA_MAX_INPUTS>(kind, p, s);
    } else {
        switch (p.n_ins) {
        case 1: return launch_chain_reduce_n<C, true, 1>(kind, p, s);
        case 2: return launch_chain_reduce_n<C, true, 2>(kind, p, s);
        case 3: return launch_chain_reduce_n<C, true, 3>(kind, p, s);
        case 4: return launch_chain_reduce_n<C, true, 4>(kind, p, s);
        case 5: return launch_chain_reduce_n<C, true, 5>(kind, p, s);
        default: return launch_chain_reduce_n<C, true, 6>(kind, p, s);
        }
    }
}

}  // namespace

int launch_chain_reduce_f32(int kind, bool vec, const ChainReduceParams& p, cudaStream_t s) {
    return vec ? launch_chain_reduce<float, true>(kind, p, s) : launch_chain_reduce<float, false>(kind, p, s);
}

int launch_chain_reduce_typed(int kind, int dt, const ChainReduceParams& p, cudaStream_t s) {
    switch (dt) {
    case TADMA_F32: return launch_typed_t<float>(kind, p, s);
    case TADMA_F16: return launch_typed_t<__half>(kind, p, s);
    default: return launch_typed_t<__nv_bfloat16>(kind, p, s);
    }
}

int launch_chain_reduce_f64(int kind, const ChainReduceParams& p, cudaStream_t s) {
    return launch_chain_reduce<double, false>(kind, p, s);
}

int launch_chain_reduce_i64(int kind, const ChainReduceParams& p, cudaStream_t s) {
    return launch_chain_reduce<int64_t, false>(kind, p, s);
}

}  // namespace tadma_b200
