// eltwise_typed.cu - compile-time typed kernels: the row-broadcast affine
// kernel, single-instruction calls, comparisons, where and one-dtype chains.
#include "eltwise_impl.cuh"

namespace tadma_b200 {
namespace {

// gelu_fast on two lanes: the same operation sequence as gelu_fast (ops.cuh),
// gelu(x) = x / (1 + 2^(-w)), w = x (K1 + K3 x^2), with the polynomial, the
// sum and the final product packed (the sign of w folded into K1, K3).
__device__ __forceinline__ unsigned long long gelu_fast2(unsigned long long x) {
    constexpr float K1 = 2.0f * 0.7978845608f * 1.4426950408889634f;
    constexpr float K3 = K1 * 0.044715f;
    const unsigned long long nw = f2_mul(x, f2_fma(f2_pack(-K3, -K3), f2_mul(x, x), f2_pack(-K1, -K1)));
    float a, b;
    f2_unpack(nw, a, b);
    float d0, d1;
    f2_unpack(f2_add(f2_pack(ex2_approx(a), ex2_approx(b)), f2_pack(1.0f, 1.0f)), d0, d1);
    return f2_mul(x, f2_pack(rcp_approx(d0), rcp_approx(d1)));
}

template <typename XT, typename OT, int ACT>
__device__ __forceinline__ void affine_row_compute(const Raw8x<XT>& raw, const float (&b)[8],
                                                   const unsigned long long (&b2)[4], float scale, OT* dst) {
    constexpr bool FAST = sizeof(OT) == 2;  // same rule as the host: fp32 compute, 16-bit store
    float v[8];
    raw8_cvt<XT>(raw, v);
    if constexpr (ACT == ACT_NONE || (ACT == ACT_GELU && FAST)) {
        const unsigned long long s2 = f2_pack(scale, scale);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            unsigned long long x = f2_add(f2_mul(f2_pack(v[2 * j], v[2 * j + 1]), s2), b2[j]);
            if constexpr (ACT == ACT_GELU) x = gelu_fast2(x);
            f2_unpack(x, v[2 * j], v[2 * j + 1]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = activation<ACT, FAST>(__fadd_rn(__fmul_rn(v[j], scale), b[j]));
    }
    raw8_store<OT>(dst, v);
}

// One CTA per tile of RB consecutive rows x 256 column vectors, no loop: all
// RB rows' loads are issued before the first row computes, and the hardware
// block scheduler hands tiles to SMs as they free up (a persistent grid-stride
// loop measured 10-15 % slower on B200 for streaming copies: its fixed share of
// work per CTA leaves the slowest SMs finishing last).
template <typename XT>
constexpr int affine_rb() { return sizeof(XT) == 2 ? 8 : 4; }

template <typename XT, typename OT, int ACT>
__global__ void __launch_bounds__(THREADS) affine_rows_kernel(const __grid_constant__ AffineRowsParams p) {
    pdl_begin();
    constexpr int RB = affine_rb<XT>();
    // blockIdx.x = row tile * column blocks + column block: the column blocks
    // of one row tile are neighbours in launch order (one contiguous region).
    const int64_t ncb = (p.ncv + THREADS - 1) / THREADS;
    const int64_t tile = (int64_t)blockIdx.x / ncb;
    const int64_t cv = ((int64_t)blockIdx.x - tile * ncb) * THREADS + threadIdx.x;
    if (cv >= p.ncv) return;
    const int64_t r0 = tile * RB;
    const XT* xcol = reinterpret_cast<const XT*>(p.x) + cv * 8;
    OT* ocol = reinterpret_cast<OT*>(p.out) + cv * 8;
    Raw8x<XT> cur[RB];
#pragma unroll
    for (int u = 0; u < RB; u++)
        if (r0 + u < p.rows) raw8_load<XT>(xcol + (r0 + u) * p.x_rs, cur[u], true);
    float b[8];
    unsigned long long b2[4];
    {
        Raw8x<XT> rb;
        raw8_load<XT>(reinterpret_cast<const XT*>(p.bias) + cv * 8, rb, false);
        raw8_cvt<XT>(rb, b);
#pragma unroll
        for (int j = 0; j < 4; j++) b2[j] = f2_pack(b[2 * j], b[2 * j + 1]);
    }
#pragma unroll
    for (int u = 0; u < RB; u++)
        if (r0 + u < p.rows) affine_row_compute<XT, OT, ACT>(cur[u], b, b2, p.scale, ocol + (r0 + u) * p.out_rs);
}

// ------------------------------------------------------- contiguous typed --
//
// Every input of one float dtype TI with a contiguous innermost dim (no
// innermost broadcast), the output of float dtype TO, fp32 compute (residual
// adds, scalings, casts, copies into and out of strided views): loads,
// conversions and stores are compile-time and only the chain is interpreted.
// The generic kernels decode dtypes per vector, which cost ~170 instructions
// per 8 elements on a 16-bit add (ncu) and held it to 4.7 TB/s.

// One-dtype chains: every operand is a TI tensor (F32 / F16 / BF16) that is
// either contiguous along the folded innermost dim (a vector operand) or
// broadcast along it (a scalar operand: a per-row mean or scale, one value
// per vector).  The host orders the operands vectors first, so the kernel
// knows at compile time which are scalars: those cost one register, not
// eight.  No operand needs a run-time dtype switch.  A thread loads U
// vectors of every operand before any compute, then runs the pre-decoded
// program: once on all 16 values with one operand, else one vector (8
// values) at a time in a rolled loop that shifts the next vector's words
// down, so the program is inlined once.
template <int NV, int NS>
constexpr int typed_steps() { return NV <= 2 ? 2 : 1; }
template <int NV, int NS>
constexpr int typed_width() { return NV + NS == 1 ? 2 * V : V; }

// Element offsets of vector vi: R1 (folded rank 1, every operand contiguous)
// needs no index decomposition; otherwise the folded dims are walked
// (outer-dim broadcasts and strided views; the innermost dim is contiguous
// or broadcast).
template <int NIN, bool R1>
__device__ __forceinline__ void typed_offsets(const ChainParams& p, int64_t vi, int64_t& oo, int64_t (&io)[NIN]) {
    if constexpr (R1) {
        oo = vi * V;
#pragma unroll
        for (int k = 0; k < NIN; k++) io[k] = vi * V;
    } else {
        offsets<NIN>(p, (uint64_t)vi * V, oo, io);
    }
}

template <typename T>
__device__ __forceinline__ float typed_scalar(const T* p) {
    if constexpr (sizeof(T) == 4) return *p;
    else if constexpr (std::is_same<T, __half>::value) return __half2float(*p);
    else return __bfloat162float(*p);
}

template <typename TI, typename TO, int NV, int NS, bool FAST, bool R1>
__global__ void __launch_bounds__(THREADS, 3) typed_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int NIN = NV + NS;
    constexpr int U = typed_steps<NV, NS>();
    constexpr int W = typed_width<NV, NS>();
    constexpr int G = W / V;  // vectors per program run
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        Raw8x<TI> raw[U][NV];
        float sc[U][NS > 0 ? NS : 1];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NIN];
                typed_offsets<NIN, R1>(p, vi, oo[u], io);
#pragma unroll
                for (int k = 0; k < NV; k++)
                    raw8_load<TI>(reinterpret_cast<const TI*>(p.in[k].base) + io[k], raw[u][k], p.in[k].streaming);
#pragma unroll
                for (int k = 0; k < NS; k++) sc[u][k] = typed_scalar<TI>(reinterpret_cast<const TI*>(p.in[NV + k].base) + io[NV + k]);
            } else {
                oo[u] = 0;
#pragma unroll
                for (int k = 0; k < NS; k++) sc[u][k] = 0.0f;
#pragma unroll
                for (int k = 0; k < NV; k++)
#pragma unroll
                    for (int w = 0; w < (int)(sizeof(raw[u][k].w) / sizeof(uint4)); w++) raw[u][k].w[w] = make_uint4(0u, 0u, 0u, 0u);
            }
        }
#pragma unroll 1
        for (int h = 0; h < U / G; h++) {
            float val[NV][W];
#pragma unroll
            for (int g = 0; g < G; g++)
#pragma unroll
                for (int k = 0; k < NV; k++) raw8_cvt<TI>(raw[g][k], &val[k][g * V]);
            float acc[W];
            // G > 1 only with one vector operand and no scalar
            run_fprog<NV, NS, W, FAST>(p.fp, acc, val, sc[0]);
#pragma unroll
            for (int g = 0; g < G; g++) {
                const int64_t vi = base + (h * G + g) * THREADS;
                if (vi < p.n) raw8_store<TO>(reinterpret_cast<TO*>(p.out) + oo[g], &acc[g * V]);
            }
            // the next vector moves to the front
#pragma unroll
            for (int u = 0; u + G < U; u++) {
                oo[u] = oo[u + G];
#pragma unroll
                for (int k = 0; k < NV; k++) raw[u][k] = raw[u + G][k];
#pragma unroll
                for (int k = 0; k < NS; k++) sc[u][k] = sc[u + G][k];
            }
        }
    }
}

// Single-instruction chains (every operator call of the eager API: a + b,
// x * s, a cast): the op is a compile-time constant as well, so no
// interpreter is inlined at all.  OP is ADD, SUB, MUL, DIV, RSUB, RDIV, MAX,
// MIN or COPY; IMM: the second operand is the immediate, else ins[1].
// Vectors per thread: 64 bytes of loads in flight for one 16-bit operand
// (4 x 16 B), as for an fp32 operand (2 x 32 B) or two 16-bit ones.
template <typename TI, int NIN>
constexpr int typed1_u() { return sizeof(TI) == 2 && NIN == 1 ? 4 : 2; }

template <typename TI, typename TO, int OP, bool IMM, bool R1>
__global__ void __launch_bounds__(THREADS) typed1_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int NIN = (OP == TADMA_OP_COPY || IMM) ? 1 : 2;
    constexpr int U = typed1_u<TI, NIN>();
    const float imm = __double2float_rn(p.prog[0].imm);
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        Raw8x<TI> raw[U][NIN];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NIN];
                typed_offsets<NIN, R1>(p, vi, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    raw8_load<TI>(reinterpret_cast<const TI*>(p.in[k].base) + io[k], raw[u][k], p.in[k].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if constexpr (OP == TADMA_OP_COPY && std::is_same<TI, TO>::value) {
                // A copy within one dtype moves the raw words (bit-exact).
                if (vi < p.n) {
                    TO* dst = reinterpret_cast<TO*>(p.out) + oo[u];
                    st_stream_v4(dst, raw[u][0].w[0]);
                    if constexpr (sizeof(TO) == 4) st_stream_v4(dst + 4, raw[u][0].w[1]);
                }
                continue;
            }
            if (vi < p.n) {
                float a[V], b[V];
                raw8_cvt<TI>(raw[u][0], a);
                if constexpr (NIN == 2) raw8_cvt<TI>(raw[u][NIN - 1], b);
#pragma unroll
                for (int j = 0; j < V; j++) {
                    if constexpr (OP != TADMA_OP_COPY) a[j] = binary(OP, a[j], IMM ? imm : b[j], 0.0f);
                }
                raw8_store<TO>(reinterpret_cast<TO*>(p.out) + oo[u], a);
            }
        }
    }
}

template <typename TI, typename TO, int OP, bool IMM>
int launch_typed1_k(const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const int64_t per_block = (int64_t)THREADS * typed1_u<TI, (OP == TADMA_OP_COPY || IMM) ? 1 : 2>();
    const int64_t want = (nvec + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    if (p.rank == 1) (void)launch_pdl(typed1_kernel<TI, TO, OP, IMM, true>, dim3(grid), dim3(THREADS), 0, s, p);
    else (void)launch_pdl(typed1_kernel<TI, TO, OP, IMM, false>, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename TI, typename TO, bool IMM>
int launch_typed1_op(int op, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (op) {
    case TADMA_OP_ADD: return launch_typed1_k<TI, TO, TADMA_OP_ADD, IMM>(p, nvec, s);
    case TADMA_OP_SUB: return launch_typed1_k<TI, TO, TADMA_OP_SUB, IMM>(p, nvec, s);
    case TADMA_OP_MUL: return launch_typed1_k<TI, TO, TADMA_OP_MUL, IMM>(p, nvec, s);
    case TADMA_OP_DIV: return launch_typed1_k<TI, TO, TADMA_OP_DIV, IMM>(p, nvec, s);
    case TADMA_OP_RSUB: return launch_typed1_k<TI, TO, TADMA_OP_RSUB, IMM>(p, nvec, s);
    case TADMA_OP_RDIV: return launch_typed1_k<TI, TO, TADMA_OP_RDIV, IMM>(p, nvec, s);
    case TADMA_OP_MAX: return launch_typed1_k<TI, TO, TADMA_OP_MAX, IMM>(p, nvec, s);
    default: return launch_typed1_k<TI, TO, TADMA_OP_MIN, IMM>(p, nvec, s);
    }
}

// Binary ops with an immediate or a second operand; casts / copies for every
// (TI, TO) pair.  Same-dtype binary ops only (TI == TO), the eager API's case.
template <typename TI, typename TO>
int launch_typed1_io(int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    if (op == TADMA_OP_COPY) return launch_typed1_k<TI, TO, TADMA_OP_COPY, false>(p, nvec, s);
    if constexpr (std::is_same<TI, TO>::value) {
        return imm ? launch_typed1_op<TI, TO, true>(op, p, nvec, s) : launch_typed1_op<TI, TO, false>(op, p, nvec, s);
    }
    return TADMA_ERR_UNSUPPORTED;
}

template <typename TI>
int launch_typed1_i(int odt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (odt) {
    case TADMA_F32: return launch_typed1_io<TI, float>(op, imm, p, nvec, s);
    case TADMA_F16: return launch_typed1_io<TI, __half>(op, imm, p, nvec, s);
    default: return launch_typed1_io<TI, __nv_bfloat16>(op, imm, p, nvec, s);
    }
}

// Comparisons of one float dtype (a tensor or an immediate on the right) into
// a bool tensor, and where(bool or u8 condition, T, T) -> T: the mask
// producers and consumers of generated graphs, typed like typed1_kernel.
__device__ __forceinline__ void store_bytes8(uint8_t* p, const float (&v)[V]) {
    uint2 w = make_uint2(0u, 0u);
#pragma unroll
    for (int j = 0; j < V; j++) {
        const uint32_t b = (v[j] != 0.0f ? 1u : 0u) << (8 * (j & 3));
        if (j < 4) w.x |= b;
        else w.y |= b;
    }
    __stcs(reinterpret_cast<uint2*>(p), w);
}

template <typename TI, int OP, bool IMM, bool R1>
__global__ void __launch_bounds__(THREADS) typed_cmp_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int U = 2;
    constexpr int NIN = IMM ? 1 : 2;
    const float imm = __double2float_rn(p.prog[0].imm);
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        Raw8x<TI> raw[U][NIN];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[NIN];
                typed_offsets<NIN, R1>(p, vi, oo[u], io);
#pragma unroll
                for (int k = 0; k < NIN; k++)
                    raw8_load<TI>(reinterpret_cast<const TI*>(p.in[k].base) + io[k], raw[u][k], p.in[k].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                float a[V], b[V];
                raw8_cvt<TI>(raw[u][0], a);
                if constexpr (!IMM) raw8_cvt<TI>(raw[u][1], b);
#pragma unroll
                for (int j = 0; j < V; j++) a[j] = binary(OP, a[j], IMM ? imm : b[j], 0.0f);
                store_bytes8(reinterpret_cast<uint8_t*>(p.out) + oo[u], a);
            }
        }
    }
}

template <typename T, bool R1>
__global__ void __launch_bounds__(THREADS) typed_where_kernel(const __grid_constant__ ChainParams p) {
    pdl_begin();
    constexpr int U = 2;
    const bool cond_bool = p.in[0].dtype == TADMA_BOOL;
    for (int64_t chunk = blockIdx.x; chunk * (THREADS * U) < p.n; chunk += gridDim.x) {
        const int64_t base = chunk * (THREADS * U) + threadIdx.x;
        uint2 c[U];
        Raw8x<T> x[U], y[U];
        int64_t oo[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                int64_t io[3];
                typed_offsets<3, R1>(p, vi, oo[u], io);
                const uint8_t* cp = reinterpret_cast<const uint8_t*>(p.in[0].base) + io[0];
                c[u] = p.in[0].streaming ? __ldcs(reinterpret_cast<const uint2*>(cp)) : *reinterpret_cast<const uint2*>(cp);
                raw8_load<T>(reinterpret_cast<const T*>(p.in[1].base) + io[1], x[u], p.in[1].streaming);
                raw8_load<T>(reinterpret_cast<const T*>(p.in[2].base) + io[2], y[u], p.in[2].streaming);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int64_t vi = base + u * THREADS;
            if (vi < p.n) {
                float fx[V], fy[V];
                raw8_cvt<T>(x[u], fx);
                raw8_cvt<T>(y[u], fy);
#pragma unroll
                for (int j = 0; j < V; j++) {
                    const uint32_t byte = ((j < 4 ? c[u].x : c[u].y) >> (8 * (j & 3))) & 0xffu;
                    const float cv = cond_bool ? (byte != 0u ? 1.0f : 0.0f) : (float)byte;
                    fx[j] = binary(TADMA_OP_WHERE, cv, fx[j], fy[j]);
                }
                raw8_store<T>(reinterpret_cast<T*>(p.out) + oo[u], fx);
            }
        }
    }
}

template <typename K>
int launch_grid2(K kernel, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const int64_t per_block = (int64_t)THREADS * 2;
    const int64_t want = (nvec + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    (void)launch_pdl(kernel, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename TI, int OP, bool IMM>
int launch_cmp_k(const ChainParams& p, int64_t nvec, cudaStream_t s) {
    return p.rank == 1 ? launch_grid2(typed_cmp_kernel<TI, OP, IMM, true>, p, nvec, s)
                       : launch_grid2(typed_cmp_kernel<TI, OP, IMM, false>, p, nvec, s);
}
template <typename TI, bool IMM>
int launch_cmp_op(int op, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (op) {
    case TADMA_OP_EQ: return launch_cmp_k<TI, TADMA_OP_EQ, IMM>(p, nvec, s);
    case TADMA_OP_NE: return launch_cmp_k<TI, TADMA_OP_NE, IMM>(p, nvec, s);
    case TADMA_OP_LT: return launch_cmp_k<TI, TADMA_OP_LT, IMM>(p, nvec, s);
    case TADMA_OP_GT: return launch_cmp_k<TI, TADMA_OP_GT, IMM>(p, nvec, s);
    case TADMA_OP_LE: return launch_cmp_k<TI, TADMA_OP_LE, IMM>(p, nvec, s);
    default: return launch_cmp_k<TI, TADMA_OP_GE, IMM>(p, nvec, s);
    }
}
template <typename TI, typename TO, int NV, int NS, bool FAST>
int launch_typed_k(const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const int64_t per_block = (int64_t)THREADS * typed_steps<NV, NS>();
    const int64_t want = (nvec + per_block - 1) / per_block;
    const int grid = (int)(want < 1 ? 1 : want > 0x7fffffff ? 0x7fffffff : want);
    // The rank-1 instance (no index walk) exists for one or two vector
    // operands without scalars: broadcasts fold to rank >= 2.
    if constexpr (NS == 0 && NV <= 2) {
        if (p.rank == 1) {
            (void)launch_pdl(typed_kernel<TI, TO, NV, NS, FAST, true>, dim3(grid), dim3(THREADS), 0, s, p);
            cudaError_t e = cudaGetLastError();
            return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
        }
    }
    (void)launch_pdl(typed_kernel<TI, TO, NV, NS, FAST, false>, dim3(grid), dim3(THREADS), 0, s, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename TI, typename TO, bool FAST, int NS>
int launch_typed_nv(int nv, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (nv) {
    case 1: return launch_typed_k<TI, TO, 1, NS, FAST>(p, nvec, s);
    case 2: return launch_typed_k<TI, TO, 2, NS, FAST>(p, nvec, s);
    case 3: return launch_typed_k<TI, TO, 3, NS, FAST>(p, nvec, s);
    case 4: return launch_typed_k<TI, TO, 4, NS, FAST>(p, nvec, s);
    case 5: if constexpr (NS <= 1) return launch_typed_k<TI, TO, 5, NS, FAST>(p, nvec, s);
            return TADMA_ERR_UNSUPPORTED;
    default: if constexpr (NS == 0) return launch_typed_k<TI, TO, 6, NS, FAST>(p, nvec, s);
             return TADMA_ERR_UNSUPPORTED;
    }
}

template <typename TI, typename TO, bool FAST>
int launch_typed_nin(int nv, int ns, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (ns) {
    case 0: return launch_typed_nv<TI, TO, FAST, 0>(nv, p, nvec, s);
    case 1: return launch_typed_nv<TI, TO, FAST, 1>(nv, p, nvec, s);
    default: return launch_typed_nv<TI, TO, FAST, 2>(nv, p, nvec, s);
    }
}

template <typename TI, typename TO>
int launch_typed_io(int nv, int ns, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    if constexpr (sizeof(TO) == 2) {
        if (fast) return launch_typed_nin<TI, TO, true>(nv, ns, p, nvec, s);
    }
    return launch_typed_nin<TI, TO, false>(nv, ns, p, nvec, s);
}

template <typename TI>
int launch_typed_i(int odt, int nv, int ns, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (odt) {
    case TADMA_F32: return launch_typed_io<TI, float>(nv, ns, fast, p, nvec, s);
    case TADMA_F16: return launch_typed_io<TI, __half>(nv, ns, fast, p, nvec, s);
    default: return launch_typed_io<TI, __nv_bfloat16>(nv, ns, fast, p, nvec, s);
    }
}

template <typename XT, typename OT, int ACT>
int launch_rows_t(const AffineRowsParams& p, cudaStream_t s) {
    const int64_t ncb = (p.ncv + THREADS - 1) / THREADS;
    const int64_t tiles = (p.rows + affine_rb<XT>() - 1) / affine_rb<XT>();
    if (ncb * tiles > 0x7fffffff) return fail(TADMA_ERR_UNSUPPORTED, "eltwise: more than 2^31 row tiles");
    cudaError_t e = launch_pdl(affine_rows_kernel<XT, OT, ACT>, dim3((unsigned)(ncb * tiles)), dim3(THREADS), 0, s, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_eltwise launch");
}

template <typename XT, typename OT>
int launch_rows_act(int act, const AffineRowsParams& p, cudaStream_t s) {
    switch (act) {
    case ACT_GELU: return launch_rows_t<XT, OT, ACT_GELU>(p, s);
    case ACT_RELU: return launch_rows_t<XT, OT, ACT_RELU>(p, s);
    case ACT_SIGMOID: return launch_rows_t<XT, OT, ACT_SIGMOID>(p, s);
    case ACT_TANH: return launch_rows_t<XT, OT, ACT_TANH>(p, s);
    default: return launch_rows_t<XT, OT, ACT_NONE>(p, s);
    }
}

}  // namespace

int launch_typed1(int idt, int odt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (idt) {
    case TADMA_F32: return launch_typed1_i<float>(odt, op, imm, p, nvec, s);
    case TADMA_F16: return launch_typed1_i<__half>(odt, op, imm, p, nvec, s);
    default: return launch_typed1_i<__nv_bfloat16>(odt, op, imm, p, nvec, s);
    }
}

// idt in {F32, F16, BF16}; the output is a bool tensor.
int launch_cmp(int idt, int op, bool imm, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (idt) {
    case TADMA_F32: return imm ? launch_cmp_op<float, true>(op, p, nvec, s) : launch_cmp_op<float, false>(op, p, nvec, s);
    case TADMA_F16: return imm ? launch_cmp_op<__half, true>(op, p, nvec, s) : launch_cmp_op<__half, false>(op, p, nvec, s);
    default:
        return imm ? launch_cmp_op<__nv_bfloat16, true>(op, p, nvec, s) : launch_cmp_op<__nv_bfloat16, false>(op, p, nvec, s);
    }
}

// dt in {F32, F16, BF16}: the branches' and the output's dtype.
int launch_where(int dt, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    const bool r1 = p.rank == 1;
    switch (dt) {
    case TADMA_F32: return r1 ? launch_grid2(typed_where_kernel<float, true>, p, nvec, s)
                              : launch_grid2(typed_where_kernel<float, false>, p, nvec, s);
    case TADMA_F16: return r1 ? launch_grid2(typed_where_kernel<__half, true>, p, nvec, s)
                              : launch_grid2(typed_where_kernel<__half, false>, p, nvec, s);
    default: return r1 ? launch_grid2(typed_where_kernel<__nv_bfloat16, true>, p, nvec, s)
                       : launch_grid2(typed_where_kernel<__nv_bfloat16, false>, p, nvec, s);
    }
}

// idt, odt in {F32, F16, BF16}; nin in {1, 2}.
int launch_typed(int idt, int odt, int nv, int ns, bool fast, const ChainParams& p, int64_t nvec, cudaStream_t s) {
    switch (idt) {
    case TADMA_F32: return launch_typed_i<float>(odt, nv, ns, fast, p, nvec, s);
    case TADMA_F16: return launch_typed_i<__half>(odt, nv, ns, fast, p, nvec, s);
    default: return launch_typed_i<__nv_bfloat16>(odt, nv, ns, fast, p, nvec, s);
    }
}

// x dtype = bias dtype in {f32, f16, bf16}; out dtype = x dtype or f32.
int launch_rows(int xdt, int odt, int act, const AffineRowsParams& p, cudaStream_t s) {
    if (xdt == TADMA_F32) return launch_rows_act<float, float>(act, p, s);
    if (xdt == TADMA_F16)
        return odt == TADMA_F16 ? launch_rows_act<__half, __half>(act, p, s) : launch_rows_act<__half, float>(act, p, s);
    return odt == TADMA_BF16 ? launch_rows_act<__nv_bfloat16, __nv_bfloat16>(act, p, s)
                             : launch_rows_act<__nv_bfloat16, float>(act, p, s);
}

}  // namespace tadma_b200
