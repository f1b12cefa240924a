// rowprog.cu - tadma_b200_row_program: per-row reductions of element chains
// and the element-wise chain that reads them, in one pass over each row.
//
// A decomposed normalisation (generated code's LayerNorm: mean, -, pow,
// mean, + eps, sqrt, /, *, +) is three kernels otherwise: two row
// reductions and a 5-operand element-wise chain, reading the row three
// times.  Here one warp owns a row at a time:
// * the row's 16-byte chunks are copied into the warp's shared-memory
//   buffer with cp.async (LDGSTS, L2-only), lane l taking chunks l, l + 32,
//   ...; the next row's copies are issued before the current row is
//   computed (two buffers per warp), so a row's load latency hides behind
//   the previous row's arithmetic without holding the row in registers;
// * each lane reads back only the chunks it copied, in the same order, so
//   cp.async.wait_group alone orders the copy before the use;
// * column operands (gamma, beta) are staged once per CTA;
// * each stage folds its chain exactly as the row reductions fold (lane l
//   visits vectors l, l + 32, ... in order, elements in order, then the
//   fixed lane butterfly; MEAN divides by cols; the post chain; rounding to
//   the stage's out dtype), so its value is the bits the separate reduction
//   call stores; the final chain is the typed kernels' pre-decoded program.
// There is no spin-wait: cp.async.wait_group is the hardware's own wait.
#include "eltwise_impl.cuh"
#include "kdiv.cuh"

namespace tadma_b200 {

constexpr int RP_MAX_RV = 2, RP_MAX_CV = 2, RP_MAX_SC = 2;
constexpr int RP_NS = RP_MAX_SC + TADMA_ROWPROG_MAX_STAGES;  // scalar slots

// A pass whose decoded program is one of the shapes a LayerNorm written out
// as separate ops produces runs as straight-line code instead of through
// the step loop (the same op bodies and roundings, so the same bits):
//   RC_COPY    x                                   (a plain mean's elements)
//   RC_SQDIFF  rnd(sqr(rnd(x - s1)))               (the variance's elements)
//   RC_LNTAIL  rnd(rnd(rnd(rnd(x - s1) / s2) * c1) + c2), the affine part
//              optional                            (the normalised output)
// rnd: none, or the rounding to fp16 / bf16 of 16-bit generated code.
constexpr int RC_GENERIC = 0, RC_COPY = 1, RC_SQDIFF = 2, RC_LNTAIL = 3, RC_LNTAIL_PLAIN = 4;
struct PassRecipe {
    int8_t kind, rnd;   // rnd: -1 none, else TADMA_F16 / TADMA_BF16
    int8_t x, s1, s2, c1, c2, pad;  // operand slots
};

struct RowStageParams {
    PassRecipe rc;
    int32_t kind;  // K_SUM, K_MAX, K_MIN
    int32_t mean;  // divide by cols
    char* out;
    int32_t out_dtype, pad;
    int64_t out_stride;
    FProg fp;
    FProg pfp;  // the post chain, pre-decoded (pfp.n == 0: none)
};

struct RowProgParams {
    int64_t rows;
    int32_t cols, nvec;  // nvec: 16-byte chunks per row
    int32_t n_stages;
    int32_t n_rv, n_cv;  // row / column operands
    int32_t fast;        // the final chain's fast-math bodies (16-bit out)
    const char* rv[RP_MAX_RV];
    int64_t rv_rs[RP_MAX_RV];  // row strides in bytes
    const char* cv[RP_MAX_CV];
    const char* sc[RP_MAX_SC];
    int32_t sc_dtype[RP_MAX_SC];
    int64_t sc_rs[RP_MAX_SC];  // row strides in elements
    RowStageParams st[TADMA_ROWPROG_MAX_STAGES];
    PassRecipe rc;  // the final pass's
    FProg fp;
    char* out;
    int64_t out_rs;  // row stride in elements
};

namespace {

template <typename TI>
__device__ __forceinline__ void cvt16(uint4 r, float (&f)[16 / sizeof(TI)]) {
    if constexpr (sizeof(TI) == 4) {
        f[0] = __uint_as_float(r.x);
        f[1] = __uint_as_float(r.y);
        f[2] = __uint_as_float(r.z);
        f[3] = __uint_as_float(r.w);
    } else {
        unpack8(r, std::is_same<TI, __half>::value ? TADMA_F16 : TADMA_BF16, f);
    }
}

// The row reductions' lane combine (reduce_state.cuh combine) with the kind
// known at run time.
__device__ __forceinline__ float combine_k(int kind, float a, float b) {
    return kind == K_SUM ? a + b : kind == K_MAX ? ((b > a || b != b) ? b : a) : ((b < a || b != b) ? b : a);
}

// The pre-decoded program of one pass (a stage's chain or the final chain)
// on a group of G chunks of the lane: step-major, so each step is
// dispatched once per G x N values and reads its operand straight from
// shared memory.  The op bodies and roundings are those of run_fprog.
// Operand slots of the kernel: row operands 0-1, column operands 2-3, row
// scalars 4-5, stage results 6-8 (RP_VEC vector slots, then RP_NS scalars).
constexpr int RP_VEC = RP_MAX_RV + RP_MAX_CV;

template <typename TI, int G>
struct RowGroup {
    static constexpr int N = 16 / (int)sizeof(TI);
    const uint4* rbuf;
    const uint4* cbuf;
    int stride, c0;  // chunks per (padded) operand buffer; chunk of u: c0 + 32 u
    __device__ __forceinline__ const uint4* base(int slot) const {
        return slot < RP_MAX_RV ? rbuf + slot * stride : cbuf + (slot - RP_MAX_RV) * stride;
    }
    // The buffers are padded to whole groups: a chunk past the row reads
    // padding, computes on it and is neither folded nor stored.
    __device__ __forceinline__ void load(int slot, int u, float (&f)[N]) const { cvt16<TI>(base(slot)[c0 + 32 * u], f); }
};

template <int NS>
__device__ __forceinline__ float scalar_slot(const float (&sv)[NS], int q) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < NS; k++)
        if (q == k) s = sv[k];
    return s;
}

#define TADMA_RU(OP)                                                                   \
    case OP: {                                                                         \
        _Pragma("unroll") for (int u = 0; u < G; u++)                                  \
            _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = funary<OP, false>(acc[u][j]); \
    } break;
#define TADMA_RUF(OP)                                                                  \
    case OP: {                                                                         \
        if (fast) {                                                                    \
            _Pragma("unroll") for (int u = 0; u < G; u++)                              \
                _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = funary<OP, true>(acc[u][j]); \
        } else {                                                                       \
            _Pragma("unroll") for (int u = 0; u < G; u++)                              \
                _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = funary<OP, false>(acc[u][j]); \
        }                                                                              \
    } break;
#define TADMA_RB(OP)                                                                   \
    case FC_BI + (OP - TADMA_OP_ADD): {                                                \
        _Pragma("unroll") for (int u = 0; u < G; u++)                                  \
            _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = binary(OP, acc[u][j], bs, bs); \
    } break;                                                                           \
    case FC_BV + (OP - TADMA_OP_ADD): {                                                \
        if (bvec) {                                                                    \
            _Pragma("unroll") for (int u = 0; u < G; u++) {                            \
                float b[N];                                                            \
                grp.load(I.b, u, b);                                                   \
                _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = binary(OP, acc[u][j], b[j], b[j]); \
            }                                                                          \
        } else {                                                                       \
            _Pragma("unroll") for (int u = 0; u < G; u++)                              \
                _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = binary(OP, acc[u][j], bs, bs); \
        }                                                                              \
    } break;
#define TADMA_RR(K, DT)                                                                \
    case FC_RND + K: {                                                                 \
        _Pragma("unroll") for (int u = 0; u < G; u++)                                  \
            _Pragma("unroll") for (int j = 0; j < N; j++) acc[u][j] = round_to(acc[u][j], DT); \
    } break;

template <typename TI, int G, int NS>
__device__ __forceinline__ void run_group(const FProg& fp, bool fast, const RowGroup<TI, G>& grp,
                                          const float (&sv)[NS], float (&acc)[G][16 / sizeof(TI)]) {
    constexpr int N = 16 / (int)sizeof(TI);
    constexpr int NV = RP_VEC;
    if (fp.acc < NV) {
#pragma unroll
        for (int u = 0; u < G; u++) grp.load(fp.acc, u, acc[u]);
    } else {
        const float s = scalar_slot<NS>(sv, fp.acc - NV);
#pragma unroll
        for (int u = 0; u < G; u++)
#pragma unroll
            for (int j = 0; j < N; j++) acc[u][j] = s;
    }
    for (int i = 0; i < fp.n; i++) {
        const FInstr I = fp.ins[i];
        const bool bvec = I.b >= 0 && I.b < NV;
        const float bs = I.b >= NV ? scalar_slot<NS>(sv, I.b - NV) : I.imm;
        switch (I.code) {
        case FC_FILL: {
#pragma unroll
            for (int u = 0; u < G; u++)
#pragma unroll
                for (int j = 0; j < N; j++) acc[u][j] = I.imm;
        } break;
            TADMA_RU(TADMA_OP_NEG)
            TADMA_RU(TADMA_OP_ABS)
            TADMA_RUF(TADMA_OP_EXP)
            TADMA_RU(TADMA_OP_LOG)
            TADMA_RU(TADMA_OP_SQRT)
            TADMA_RU(TADMA_OP_SIN)
            TADMA_RU(TADMA_OP_COS)
            TADMA_RU(TADMA_OP_TAN)
            TADMA_RU(TADMA_OP_ASIN)
            TADMA_RU(TADMA_OP_ACOS)
            TADMA_RU(TADMA_OP_ATAN)
            TADMA_RU(TADMA_OP_ASINH)
            TADMA_RU(TADMA_OP_ACOSH)
            TADMA_RU(TADMA_OP_ATANH)
            TADMA_RU(TADMA_OP_ERF)
            TADMA_RU(TADMA_OP_RELU)
            TADMA_RUF(TADMA_OP_SIGMOID)
            TADMA_RU(TADMA_OP_TANH)
            TADMA_RUF(TADMA_OP_GELU)
            TADMA_RU(TADMA_OP_NOT)
            TADMA_RB(TADMA_OP_ADD)
            TADMA_RB(TADMA_OP_SUB)
            TADMA_RB(TADMA_OP_MUL)
            TADMA_RB(TADMA_OP_DIV)
            TADMA_RB(TADMA_OP_POW)
            TADMA_RB(TADMA_OP_RSUB)
            TADMA_RB(TADMA_OP_RDIV)
            TADMA_RB(TADMA_OP_MAX)
            TADMA_RB(TADMA_OP_MIN)
            TADMA_RB(TADMA_OP_EQ)
            TADMA_RB(TADMA_OP_NE)
            TADMA_RB(TADMA_OP_LT)
            TADMA_RB(TADMA_OP_GT)
            TADMA_RB(TADMA_OP_LE)
            TADMA_RB(TADMA_OP_GE)
            TADMA_RB(TADMA_OP_AND)
            TADMA_RB(TADMA_OP_OR)
            TADMA_RB(TADMA_OP_XOR)
            TADMA_RB(TADMA_OP_LAND)
            TADMA_RB(TADMA_OP_LOR)
        case FC_WHERE: {
            const bool cvec = I.c >= 0 && I.c < NV;
            const float cs = I.c >= NV ? scalar_slot<NS>(sv, I.c - NV) : I.imm;
#pragma unroll
            for (int u = 0; u < G; u++) {
                float b[N], c[N];
                if (bvec) grp.load(I.b, u, b);
                if (cvec) grp.load(I.c, u, c);
#pragma unroll
                for (int j = 0; j < N; j++) acc[u][j] = acc[u][j] != 0.0f ? (bvec ? b[j] : bs) : (cvec ? c[j] : cs);
            }
        } break;
        case FC_SQR: {
#pragma unroll
            for (int u = 0; u < G; u++)
#pragma unroll
                for (int j = 0; j < N; j++) acc[u][j] = __fmul_rn(acc[u][j], acc[u][j]);
        } break;
        case FC_DIVK: {
            const KnownDivisor kd{I.imm, fp.ins[i + 1].imm, true};
            i++;  // the reciprocal's step
#pragma unroll
            for (int u = 0; u < G; u++) {
                bool fast = true;
#pragma unroll
                for (int j = 0; j < N; j++) fast = fast & kdiv_in_range(acc[u][j]);
                if (fast) {
#pragma unroll
                    for (int j = 0; j < N; j++) acc[u][j] = kdiv_fast(acc[u][j], kd);
                } else {
#pragma unroll
                    for (int j = 0; j < N; j++) acc[u][j] = __fdiv_rn(acc[u][j], kd.b);
                }
            }
        } break;
            TADMA_RR(0, TADMA_F16)
            TADMA_RR(1, TADMA_BF16)
            TADMA_RR(2, TADMA_I64)
            TADMA_RR(3, TADMA_I32)
            TADMA_RR(4, TADMA_U8)
            TADMA_RR(5, TADMA_BOOL)
            TADMA_RR(6, TADMA_I8)
        default:
            break;
        }
    }
}

#undef TADMA_RU
#undef TADMA_RUF
#undef TADMA_RB
#undef TADMA_RR

template <int RD>
__device__ __forceinline__ float rc_rnd(float v) {
    if constexpr (RD < 0) return v;
    else return round_to(v, RD);
}

template <typename TI, int G, int RD, int NS>
__device__ __forceinline__ void run_recipe_r(const PassRecipe& rc, const RowGroup<TI, G>& grp, const float (&sv)[NS],
                                             float (&acc)[G][16 / sizeof(TI)]) {
    constexpr int N = 16 / (int)sizeof(TI);
#pragma unroll
    for (int u = 0; u < G; u++) grp.load(rc.x, u, acc[u]);
    if (rc.kind == RC_COPY) return;
    const float s1 = scalar_slot<NS>(sv, rc.s1 - RP_VEC);
    if (rc.kind == RC_SQDIFF) {
#pragma unroll
        for (int u = 0; u < G; u++)
#pragma unroll
            for (int j = 0; j < N; j++) {
                const float d = rc_rnd<RD>(binary(TADMA_OP_SUB, acc[u][j], s1, s1));
                acc[u][j] = rc_rnd<RD>(__fmul_rn(d, d));
            }
        return;
    }
    const float s2 = scalar_slot<NS>(sv, rc.s2 - RP_VEC);
    // The division by the row's s2: its reciprocal once, then the fused
    // sequence of kdiv.cuh for the group when every dividend is inside its
    // range (the same bits as the IEEE division, which the group takes
    // otherwise).
    const KnownDivisor kd = known_divisor(s2);
    bool fast = kd.ok;
#pragma unroll
    for (int u = 0; u < G; u++)
#pragma unroll
        for (int j = 0; j < N; j++) {
            acc[u][j] = rc_rnd<RD>(binary(TADMA_OP_SUB, acc[u][j], s1, s1));
            fast = fast & kdiv_in_range(acc[u][j]);
        }
    // chunk by chunk (one chunk's temporaries live at a time)
#pragma unroll
    for (int u = 0; u < G; u++) {
        if (fast) {
#pragma unroll
            for (int j = 0; j < N; j++) acc[u][j] = rc_rnd<RD>(kdiv_fast(acc[u][j], kd));
        } else {
#pragma unroll
            for (int j = 0; j < N; j++) acc[u][j] = rc_rnd<RD>(binary(TADMA_OP_DIV, acc[u][j], s2, s2));
        }
        if (rc.kind == RC_LNTAIL) {
            float g[N], b[N];
            grp.load(rc.c1, u, g);
            grp.load(rc.c2, u, b);
#pragma unroll
            for (int j = 0; j < N; j++) {
                const float t = rc_rnd<RD>(binary(TADMA_OP_MUL, acc[u][j], g[j], g[j]));
                acc[u][j] = rc_rnd<RD>(binary(TADMA_OP_ADD, t, b[j], b[j]));
            }
        }
    }
}

template <typename TI, int G, int NS>
__device__ __forceinline__ void run_recipe(const PassRecipe& rc, const RowGroup<TI, G>& grp, const float (&sv)[NS],
                                           float (&acc)[G][16 / sizeof(TI)]) {
    if (rc.rnd == TADMA_F16) run_recipe_r<TI, G, TADMA_F16, NS>(rc, grp, sv, acc);
    else if (rc.rnd == TADMA_BF16) run_recipe_r<TI, G, TADMA_BF16, NS>(rc, grp, sv, acc);
    else run_recipe_r<TI, G, -1, NS>(rc, grp, sv, acc);
}

// Chunk c of the final pass's output row.
template <typename TO, int N>
__device__ __forceinline__ void store_chunk(TO* orow, int c, const float (&a)[N]) {
    if constexpr (sizeof(TO) == 4) {
#pragma unroll
        for (int j = 0; j < N; j += 4)
            st_stream_v4(orow + c * N + j, make_uint4(__float_as_uint(a[j]), __float_as_uint(a[j + 1]), __float_as_uint(a[j + 2]),
                                                      __float_as_uint(a[j + 3])));
    } else if constexpr (N == 8) {
        st_stream_v4(orow + c * N, pack8(a, std::is_same<TO, __half>::value ? TADMA_F16 : TADMA_BF16));
    } else {
        // 16-bit out, fp32 rows: 4 values, 8 bytes
        const int dt = std::is_same<TO, __half>::value ? TADMA_F16 : TADMA_BF16;
        float f8[8] = {a[0], a[1], a[2], a[3], 0.0f, 0.0f, 0.0f, 0.0f};
        const uint4 w = pack8(f8, dt);
        __stcs(reinterpret_cast<uint2*>(orow + c * N), make_uint2(w.x, w.y));
    }
}

// One pass of a recipe-only program over the lane's G chunks, chunk by
// chunk: chunk u is computed (the op bodies and roundings of run_recipe_r),
// then folded into acc_s (a stage, in chunk order) or stored (the final
// pass), so only one chunk's temporaries are live.  RK: the recipe, RD its
// rounding.
template <typename TI, typename TO, int G, int RK, int RD>
__device__ __forceinline__ void recipe_pass(const PassRecipe& rc, const RowGroup<TI, G>& grp, float s1, float s2,
                                            const KnownDivisor& kd, bool final_pass, int kind, float& acc_s, TO* orow) {
    constexpr int N = 16 / (int)sizeof(TI);
    // the lane's first chunk of each operand; chunk u is 32 u further
    const uint4* xb = grp.base(rc.x) + grp.c0;
    const uint4* gb = grp.base(RK == RC_LNTAIL ? rc.c1 : rc.x) + grp.c0;
    const uint4* bb = grp.base(RK == RC_LNTAIL ? rc.c2 : rc.x) + grp.c0;
#pragma unroll
    for (int u = 0; u < G; u++) {
        float a[N];
        cvt16<TI>(xb[32 * u], a);
        if constexpr (RK == RC_SQDIFF) {
#pragma unroll
            for (int j = 0; j < N; j++) {
                const float d = rc_rnd<RD>(binary(TADMA_OP_SUB, a[j], s1, s1));
                a[j] = rc_rnd<RD>(__fmul_rn(d, d));
            }
        } else if constexpr (RK == RC_LNTAIL || RK == RC_LNTAIL_PLAIN) {
            bool fast = kd.ok;
#pragma unroll
            for (int j = 0; j < N; j++) {
                a[j] = rc_rnd<RD>(binary(TADMA_OP_SUB, a[j], s1, s1));
                fast = fast & kdiv_in_range(a[j]);
            }
            if (fast) {
#pragma unroll
                for (int j = 0; j < N; j++) a[j] = rc_rnd<RD>(kdiv_fast(a[j], kd));
            } else {
#pragma unroll
                for (int j = 0; j < N; j++) a[j] = rc_rnd<RD>(binary(TADMA_OP_DIV, a[j], s2, s2));
            }
            if constexpr (RK == RC_LNTAIL) {
                float g[N], b[N];
                cvt16<TI>(gb[32 * u], g);
                cvt16<TI>(bb[32 * u], b);
#pragma unroll
                for (int j = 0; j < N; j++) a[j] = rc_rnd<RD>(binary(TADMA_OP_ADD, rc_rnd<RD>(binary(TADMA_OP_MUL, a[j], g[j], g[j])), b[j], b[j]));
            }
        }
        if (final_pass) {
            store_chunk<TO, N>(orow, grp.c0 + 32 * u, a);
        } else if (kind == K_SUM) {
#pragma unroll
            for (int j = 0; j < N; j++) acc_s = acc_s + a[j];
        } else if (kind == K_MAX) {
#pragma unroll
            for (int j = 0; j < N; j++) acc_s = fmax_nan(acc_s, a[j]);
        } else {
#pragma unroll
            for (int j = 0; j < N; j++) acc_s = fmin_nan(acc_s, a[j]);
        }
    }
}

// The rounding of a recipe-only kernel's passes: none, or (16-bit rows) the
// rows' own type; the host sends programs with other roundings to the
// generic kernel (launch_rp_t), so each kernel holds one or two
// variants of each pass.
template <typename TI>
constexpr int rp_own_rnd() { return sizeof(TI) == 4 ? -1 : std::is_same<TI, __half>::value ? TADMA_F16 : TADMA_BF16; }

template <typename TI, typename TO, int G, int RK>
__device__ __forceinline__ void recipe_pass_r(const PassRecipe& rc, const RowGroup<TI, G>& grp, float s1, float s2,
                                              const KnownDivisor& kd, bool final_pass, int kind, float& acc_s, TO* orow) {
    if constexpr (rp_own_rnd<TI>() >= 0) {
        if (rc.rnd >= 0) {
            recipe_pass<TI, TO, G, RK, rp_own_rnd<TI>()>(rc, grp, s1, s2, kd, final_pass, kind, acc_s, orow);
            return;
        }
    }
    recipe_pass<TI, TO, G, RK, -1>(rc, grp, s1, s2, kd, final_pass, kind, acc_s, orow);
}

// Chunks of one operand buffer in shared memory: the row's, padded to whole
// groups of G chunks per lane.
__host__ __device__ constexpr int rp_stride(int nvec, int G) { return (nvec + 32 * G - 1) / (32 * G) * (32 * G); }

// RONLY: every pass is a recipe (the step loop is not compiled in, so a
// group can hold the lane's whole row: G = its chunk count; passes run chunk
// by chunk in at most 64 registers, four CTAs per SM where shared memory
// allows).
template <typename TI, typename TO, int G, bool RONLY>
__global__ void __launch_bounds__(THREADS, RONLY ? 4 : 3) rowprog_kernel(const __grid_constant__ RowProgParams p) {
    pdl_begin();
    constexpr int N = 16 / (int)sizeof(TI);
    extern __shared__ uint4 rp_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nvec = p.nvec;
    const int stride = rp_stride(nvec, G);
    const int nrv = p.n_rv, ncv = p.n_cv;
    uint4* colbuf = rp_smem;                                           // ncv x stride
    uint4* wbuf = rp_smem + ncv * stride + warp * (2 * nrv * stride);  // 2 buffers x nrv x stride
    for (int i = threadIdx.x; i < ncv * nvec; i += blockDim.x)
        colbuf[(i / nvec) * stride + i % nvec] = *reinterpret_cast<const uint4*>(p.cv[i / nvec] + (int64_t)(i % nvec) * 16);
    __syncthreads();

    const int64_t nw = (int64_t)gridDim.x * (THREADS / 32);
    int64_t row = (int64_t)blockIdx.x * (THREADS / 32) + warp;
    auto issue = [&](int64_t r, int b) {
        for (int k = 0; k < nrv; k++) {
            const char* src = p.rv[k] + r * p.rv_rs[k];
            uint4* dst = wbuf + (b * nrv + k) * stride;
            if constexpr (RONLY) {
                // nvec == 32 G: the lane's G chunks at fixed offsets
#pragma unroll
                for (int u = 0; u < G; u++) cp_async16(dst + lane + 32 * u, src + (int64_t)(lane + 32 * u) * 16);
            } else {
                for (int c = lane; c < nvec; c += 32) cp_async16(dst + c, src + (int64_t)c * 16);
            }
        }
        cp_async_commit();
    };
    // chunks of this lane: lane, lane + 32, ...; groups of G of them
    const int nchunk = lane < nvec ? (nvec - lane + 31) / 32 : 0;
    const int ngroups = stride / (32 * G);
    if (row < p.rows) issue(row, 0);
    for (int b = 0; row < p.rows; row += nw, b ^= 1) {
        if (row + nw < p.rows) {
            issue(row + nw, b ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        RowGroup<TI, G> grp{wbuf + b * nrv * stride, colbuf, stride, 0};
        // scalar slots: the row scalars, then the stage results
        float sv[RP_NS];
#pragma unroll
        for (int k = 0; k < RP_NS; k++) sv[k] = 0.0f;
#pragma unroll
        for (int k = 0; k < RP_MAX_SC; k++)
            if (p.sc[k]) sv[k] = load_as<float>(p.sc[k], p.sc_dtype[k], row * p.sc_rs[k]);

        // passes 0 .. n_stages - 1: the stages; pass n_stages: the final chain
#pragma unroll 1
        for (int s = 0; s <= p.n_stages; s++) {
            const bool final_pass = s == p.n_stages;
            const FProg& fp = final_pass ? p.fp : p.st[s].fp;
            const PassRecipe& rc = final_pass ? p.rc : p.st[s].rc;
            const int kind = final_pass ? K_SUM : p.st[s].kind;
            float acc_s = kind == K_SUM ? 0.0f : kind == K_MAX ? -INFINITY : INFINITY;
            TO* orow = reinterpret_cast<TO*>(p.out) + row * p.out_rs;
            if constexpr (RONLY) {
                // one group: the lane's G chunks, lane, lane + 32, ...
                grp.c0 = lane;
                const float s1 = rc.kind >= RC_SQDIFF ? scalar_slot<RP_NS>(sv, rc.s1 - RP_VEC) : 0.0f;
                const float s2 = rc.kind >= RC_LNTAIL ? scalar_slot<RP_NS>(sv, rc.s2 - RP_VEC) : 1.0f;
                KnownDivisor kd{1.0f, 1.0f, true};
                if (rc.kind >= RC_LNTAIL) kd = known_divisor(s2);
                switch (rc.kind) {
                case RC_COPY: recipe_pass<TI, TO, G, RC_COPY, -1>(rc, grp, s1, s2, kd, final_pass, kind, acc_s, orow); break;
                case RC_SQDIFF: recipe_pass_r<TI, TO, G, RC_SQDIFF>(rc, grp, s1, s2, kd, final_pass, kind, acc_s, orow); break;
                case RC_LNTAIL: recipe_pass_r<TI, TO, G, RC_LNTAIL>(rc, grp, s1, s2, kd, final_pass, kind, acc_s, orow); break;
                default: recipe_pass_r<TI, TO, G, RC_LNTAIL_PLAIN>(rc, grp, s1, s2, kd, final_pass, kind, acc_s, orow); break;
                }
            } else {
#pragma unroll 1
                for (int g = 0; g < ngroups; g++) {
                    grp.c0 = lane + 32 * G * g;
                    const int nval = nchunk - G * g;  // chunks of this group inside the row (may be <= 0 or > G)
                    float a[G][N];
                    if (rc.kind != RC_GENERIC) run_recipe<TI, G, RP_NS>(rc, grp, sv, a);
                    else run_group<TI, G, RP_NS>(fp, final_pass && p.fast, grp, sv, a);
                    if (!final_pass) {
                        // the row reductions' per-element fold, in chunk order
                        if (kind == K_SUM) {
#pragma unroll
                            for (int u = 0; u < G; u++)
                                if (u < nval)
#pragma unroll
                                    for (int j = 0; j < N; j++) acc_s = acc_s + a[u][j];
                        } else if (kind == K_MAX) {
#pragma unroll
                            for (int u = 0; u < G; u++)
                                if (u < nval)
#pragma unroll
                                    for (int j = 0; j < N; j++) acc_s = fmax_nan(acc_s, a[u][j]);
                        } else {
#pragma unroll
                            for (int u = 0; u < G; u++)
                                if (u < nval)
#pragma unroll
                                    for (int j = 0; j < N; j++) acc_s = fmin_nan(acc_s, a[u][j]);
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < G; u++)
                            if (u < nval) store_chunk<TO, N>(orow, grp.c0 + 32 * u, a[u]);
                    }
                }
            }
            if (final_pass) break;
            const RowStageParams& st = p.st[s];
            if (kind == K_SUM) {
                // the fixed-order butterfly of the row reductions; fp32
                // addition is commutative, so lane order needs no select
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc_s = acc_s + __shfl_xor_sync(0xffffffffu, acc_s, o);
            } else {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float t = __shfl_xor_sync(0xffffffffu, acc_s, o);
                    acc_s = (lane & o) ? combine_k(kind, t, acc_s) : combine_k(kind, acc_s, t);
                }
            }
            float v = acc_s;
            if (st.mean) v = v / (float)p.cols;
            if (st.pfp.n) {
                const float in[1][1] = {{v}};
                float r[1];
                run_fprog<1, 1, false>(st.pfp, r, in);
                v = r[0];
            }
            v = round_to(v, st.out_dtype);
            if (lane == 0) store_from(st.out, st.out_dtype, row * st.out_stride, v);
            if (s == 0) sv[RP_MAX_SC + 0] = v;
            else if (s == 1) sv[RP_MAX_SC + 1] = v;
            else sv[RP_MAX_SC + 2] = v;
        }
        __syncwarp();  // every lane is done with buffer b before it is refilled
    }
    cp_async_wait<0>();
}

template <typename TI, typename TO, int G, bool RONLY = false>
int launch_rp_g(const RowProgParams& p, cudaStream_t s) {
    const void* fn = (const void*)rowprog_kernel<TI, TO, G, RONLY>;
    const int stride = rp_stride(p.nvec, G);
    const size_t smem = (size_t)(p.n_cv * stride + (THREADS / 32) * 2 * p.n_rv * stride) * 16;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_row_program smem attribute");
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, THREADS, smem);
    if (e != cudaSuccess) return cuda_fail(e, "tadma_b200_row_program occupancy");
    if (per_sm < 1) return fail(TADMA_ERR_UNSUPPORTED, "tadma_b200_row_program: rows do not fit shared memory");
    const int64_t want = (p.rows + THREADS / 32 - 1) / (THREADS / 32);
    const int64_t cap = (int64_t)sm_count() * per_sm;
    const int grid = (int)(want < cap ? want : cap);
    e = launch_pdl(rowprog_kernel<TI, TO, G, RONLY>, dim3(grid), dim3(THREADS), smem, s, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_row_program launch");
}

// Chunks per program run: 16-bit rows 2 (16 values); fp32 rows 4 (16
// values) when that pads the lane's chunks no more than 2 (8 values) does.
template <typename TI, typename TO>
int launch_rp_t(const RowProgParams& p, cudaStream_t s) {
    // every pass a recipe and every lane the same whole chunks: one group
    // holds the lane's row (512 / 768 / 1024 values)
    // (passes rounded, if at all, to the rows' own 16-bit type)
    auto rnd_ok = [](const PassRecipe& rc) { return rc.kind == RC_COPY || rc.rnd < 0 || rc.rnd == rp_own_rnd<TI>(); };
    bool all_rc = p.rc.kind != RC_GENERIC && rnd_ok(p.rc);
    for (int k = 0; k < p.n_stages; k++) all_rc = all_rc && p.st[k].rc.kind != RC_GENERIC && rnd_ok(p.st[k].rc);
    if (all_rc && p.nvec % 32 == 0) {
        const int per_lane = p.nvec / 32;
        constexpr int N = 16 / (int)sizeof(TI);
        if (per_lane * N == 16) return launch_rp_g<TI, TO, 16 / N, true>(p, s);
        if (per_lane * N == 24) return launch_rp_g<TI, TO, 24 / N, true>(p, s);
        if (per_lane * N == 32) return launch_rp_g<TI, TO, 32 / N, true>(p, s);
    }
    if constexpr (sizeof(TI) == 4) {
        const int per_lane = (p.nvec + 31) / 32;
        auto waste = [&](int g) { return (per_lane + g - 1) / g * g - per_lane; };
        if (waste(4) <= waste(2)) return launch_rp_g<TI, TO, 4>(p, s);
    }
    return launch_rp_g<TI, TO, 2>(p, s);
}

template <typename TI>
int launch_rp_i(int odt, const RowProgParams& p, cudaStream_t s) {
    if (odt == TADMA_F32) return launch_rp_t<TI, float>(p, s);
    if (odt == TADMA_F16) return launch_rp_t<TI, __half>(p, s);
    return launch_rp_t<TI, __nv_bfloat16>(p, s);
}

// The recipe of a decoded pass program (RC_GENERIC when none fits).  Slots:
// 0-1 row operands, 2-3 column operands, 4+ scalars.
PassRecipe match_recipe(const FProg& fp) {
    PassRecipe rc{};
    rc.kind = RC_GENERIC;
    rc.rnd = -1;
    if (fp.acc < 0 || fp.acc >= RP_MAX_RV) return rc;
    rc.x = (int8_t)fp.acc;
    int i = 0, rnd = -2;  // -2: not yet seen
    // one step of code `code` (operand class checked by the caller), then an
    // optional rounding, the same for every step
    auto step = [&](int code) -> const FInstr* {
        if (i >= fp.n || fp.ins[i].code != code) return nullptr;
        const FInstr* f = &fp.ins[i++];
        int r = -1;
        if (i < fp.n && fp.ins[i].code >= FC_RND && fp.ins[i].code <= FC_RND + 1) r = fp.ins[i++].code == FC_RND ? TADMA_F16 : TADMA_BF16;
        if (rnd == -2) rnd = r;
        return r == rnd ? f : nullptr;
    };
    auto scalar = [](const FInstr* f) { return f && f->b >= RP_VEC; };
    auto column = [](const FInstr* f) { return f && f->b >= RP_MAX_RV && f->b < RP_VEC; };
    if (fp.n == 0) {
        rc.kind = RC_COPY;
        return rc;
    }
    const FInstr* sub = step(FC_BV + (TADMA_OP_SUB - TADMA_OP_ADD));
    if (!scalar(sub)) return rc;
    rc.s1 = sub->b;
    if (i < fp.n && fp.ins[i].code == FC_SQR) {
        if (step(FC_SQR) && i == fp.n) {
            rc.kind = RC_SQDIFF;
            rc.rnd = (int8_t)rnd;
        }
        return rc;
    }
    const FInstr* div = step(FC_BV + (TADMA_OP_DIV - TADMA_OP_ADD));
    if (!scalar(div)) return rc;
    rc.s2 = div->b;
    if (i == fp.n) {
        rc.kind = RC_LNTAIL_PLAIN;
        rc.rnd = (int8_t)rnd;
        return rc;
    }
    const FInstr* mul = step(FC_BV + (TADMA_OP_MUL - TADMA_OP_ADD));
    const FInstr* add = column(mul) ? step(FC_BV + (TADMA_OP_ADD - TADMA_OP_ADD)) : nullptr;
    if (!column(mul) || !column(add) || i != fp.n) return rc;
    rc.c1 = mul->b;
    rc.c2 = add->b;
    rc.kind = RC_LNTAIL;
    rc.rnd = (int8_t)rnd;
    return rc;
}

}  // namespace
}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_row_program(const tadma_row_program* rp, void* stream) {
    if (!rp) return fail(TADMA_ERR_INVALID, "rp is NULL");
    const int64_t rows = rp->rows, cols = rp->cols;
    if (rows < 0 || cols < 1) return fail(TADMA_ERR_INVALID, "rows must be >= 0 and cols >= 1");
    if (rp->n_ins < 1 || rp->n_ins > TADMA_MAX_INPUTS) return fail(TADMA_ERR_INVALID, "n_ins out of range [1, 6]");
    if (rp->n_stages < 0 || rp->n_stages > TADMA_ROWPROG_MAX_STAGES) return fail(TADMA_ERR_INVALID, "n_stages out of range [0, 3]");
    if (rp->n_instr < 0 || rp->n_instr > TADMA_MAX_INSTR) return fail(TADMA_ERR_INVALID, "n_instr out of range [0, 16]");
    if (rp->compute != TADMA_COMPUTE_F32 && rp->compute != TADMA_COMPUTE_F32_PRECISE)
        return fail(TADMA_ERR_UNSUPPORTED, "row programs compute in fp32");
    std::string err = check_tensor(&rp->out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    const tadma_tensor& o = rp->out;
    if (o.rank != 2 || o.dims[0] != rows || o.dims[1] != cols || (cols > 1 && o.strides[1] != 1))
        return fail(TADMA_ERR_INVALID, "out must be a {rows, cols} view with unit column stride");
    if (o.dtype != TADMA_F32 && o.dtype != TADMA_F16 && o.dtype != TADMA_BF16)
        return fail(TADMA_ERR_UNSUPPORTED, "out dtype must be F32, F16 or BF16");
    const int n_ops = rp->n_ins + rp->n_stages;
    auto valid_prog = [&](const tadma_instr* prog, int n, int avail) -> bool {
        for (int i = 0; i < n; i++) {
            const tadma_instr& I = prog[i];
            const bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
            if (needs_b && !(I.b == TADMA_SRC_IMM || (I.b >= 0 && I.b < avail))) return false;
            if (I.op == TADMA_OP_WHERE && !(I.c == TADMA_SRC_IMM || (I.c >= 0 && I.c < avail))) return false;
            if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return false;
        }
        return true;
    };
    if (rp->acc < 0 || rp->acc >= n_ops || !valid_prog(rp->prog, rp->n_instr, n_ops))
        return fail(TADMA_ERR_INVALID, "prog: operand out of range or bad round_dtype");
    if (rows == 0) return TADMA_OK;

    // Classify the operands: row (cs = 1), column (rows dim 1 or rs = 0,
    // cs = 1) or row scalar (cols dim 1 or cs = 0).
    RowProgParams p{};
    p.rows = rows;
    p.cols = (int32_t)cols;
    int slot_of[TADMA_MAX_INPUTS + TADMA_ROWPROG_MAX_STAGES];
    int nrv = 0, ncv = 0, nsc = 0, ti = -1;
    int kind_of[TADMA_MAX_INPUTS];  // 0 row, 1 column, 2 scalar
    for (int k = 0; k < rp->n_ins; k++) {
        const tadma_tensor& t = rp->ins[k];
        err = check_tensor(&t, "ins[k]");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (t.rank != 2 || (t.dims[0] != rows && t.dims[0] != 1) || (t.dims[1] != cols && t.dims[1] != 1))
            return fail(TADMA_ERR_INVALID, "ins[k] must be a rank-2 view of {rows, cols} (dims may be 1)");
        const int64_t cs = t.dims[1] == 1 ? 0 : t.strides[1];
        if (cs == 1 && cols > 1) {
            if (t.dtype != TADMA_F32 && t.dtype != TADMA_F16 && t.dtype != TADMA_BF16)
                return fail(TADMA_ERR_UNSUPPORTED, "row / column operands must be F32, F16 or BF16");
            if (ti >= 0 && t.dtype != ti) return fail(TADMA_ERR_UNSUPPORTED, "row / column operands must share one dtype");
            ti = t.dtype;
            // a column operand repeats one row: stride 0, or a single row over several
            kind_of[k] = (t.strides[0] == 0 || (t.dims[0] == 1 && rows > 1)) ? 1 : 0;
        } else if (cs == 0) {
            if (t.dtype != TADMA_F32 && t.dtype != TADMA_F16 && t.dtype != TADMA_BF16 && t.dtype != TADMA_F64)
                return fail(TADMA_ERR_UNSUPPORTED, "row scalars must be float");
            kind_of[k] = 2;
        } else {
            return fail(TADMA_ERR_UNSUPPORTED, "ins[k]: the column stride must be 1 or 0");
        }
        if (kind_of[k] == 0 && nrv == RP_MAX_RV) return fail(TADMA_ERR_UNSUPPORTED, "more than 2 row operands");
        if (kind_of[k] == 1 && ncv == RP_MAX_CV) return fail(TADMA_ERR_UNSUPPORTED, "more than 2 column operands");
        if (kind_of[k] == 2 && nsc == RP_MAX_SC) return fail(TADMA_ERR_UNSUPPORTED, "more than 2 row scalars");
        if (kind_of[k] == 0) nrv++;
        else if (kind_of[k] == 1) ncv++;
        else nsc++;
    }
    if (nrv == 0 || ti < 0) return fail(TADMA_ERR_UNSUPPORTED, "a row program needs a row operand");
    const int es = dtype_size(ti);
    const int N = 16 / es;
    if (cols % N != 0 || cols > 32 * 8 * N) return fail(TADMA_ERR_UNSUPPORTED, "cols must be a multiple of 16 bytes and at most 256 chunks");
    p.nvec = (int32_t)(cols / N);
    int irv = 0, icv = 0, isc = 0;
    for (int k = 0; k < rp->n_ins; k++) {
        const tadma_tensor& t = rp->ins[k];
        const int64_t rs = t.dims[0] == 1 ? 0 : t.strides[0];
        if (kind_of[k] == 0) {
            if ((uintptr_t)t.data % 16 || (rs * es) % 16) return fail(TADMA_ERR_UNSUPPORTED, "row operands need 16-byte aligned rows");
            p.rv[irv] = (const char*)t.data;
            p.rv_rs[irv] = rs * es;
            slot_of[k] = irv++;
        } else if (kind_of[k] == 1) {
            if ((uintptr_t)t.data % 16) return fail(TADMA_ERR_UNSUPPORTED, "column operands must be 16-byte aligned");
            p.cv[icv] = (const char*)t.data;
            slot_of[k] = RP_MAX_RV + icv++;
        } else {
            p.sc[isc] = (const char*)t.data;
            p.sc_dtype[isc] = t.dtype;
            p.sc_rs[isc] = rs;
            slot_of[k] = RP_VEC + isc++;
        }
    }
    for (int s = 0; s < rp->n_stages; s++) slot_of[rp->n_ins + s] = RP_VEC + RP_MAX_SC + s;
    p.n_rv = nrv;
    p.n_cv = ncv;

    p.n_stages = rp->n_stages;
    for (int s = 0; s < rp->n_stages; s++) {
        const tadma_row_stage& S = rp->stages[s];
        RowStageParams& st = p.st[s];
        const int avail = rp->n_ins + s;  // a stage reads earlier stages only
        if (S.op != TADMA_REDUCE_SUM && S.op != TADMA_REDUCE_MEAN && S.op != TADMA_REDUCE_MAX && S.op != TADMA_REDUCE_MIN)
            return fail(TADMA_ERR_UNSUPPORTED, "stage op must be SUM, MEAN, MAX or MIN");
        if (S.n_instr < 0 || S.n_instr > TADMA_MAX_INSTR || S.n_post < 0 || S.n_post > TADMA_MAX_INSTR)
            return fail(TADMA_ERR_INVALID, "stage program length out of range [0, 16]");
        if (S.acc < 0 || S.acc >= avail || !valid_prog(S.prog, S.n_instr, avail))
            return fail(TADMA_ERR_INVALID, "stage program: operand out of range or bad round_dtype");
        for (int i = 0; i < S.n_post; i++) {
            const tadma_instr& I = S.post[i];
            const bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
            if (I.op == TADMA_OP_WHERE || (needs_b && I.b != TADMA_SRC_IMM))
                return fail(TADMA_ERR_INVALID, "stage post: operands must be immediates");
            if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return fail(TADMA_ERR_INVALID, "bad round_dtype in post");
        }
        // the post chain on the stage's value (operand 0), immediates only
        if (!decode_fprog(S.post, S.n_post, 1, st.pfp))
            return fail(TADMA_ERR_UNSUPPORTED, "stage post step has no typed code");
        err = check_tensor(&S.out, "stage out");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (S.out.rank != 1 || S.out.dims[0] != rows) return fail(TADMA_ERR_INVALID, "stage out must be a {rows} view");
        st.out = (char*)S.out.data;
        st.out_dtype = S.out.dtype;
        st.out_stride = S.out.strides[0];
        st.kind = S.op == TADMA_REDUCE_MAX ? K_MAX : S.op == TADMA_REDUCE_MIN ? K_MIN : K_SUM;
        st.mean = S.op == TADMA_REDUCE_MEAN;
        if (!decode_fprog(S.prog, S.n_instr, avail, st.fp, slot_of))
            return fail(TADMA_ERR_UNSUPPORTED, "stage program step has no typed code");
        st.fp.acc = slot_of[S.acc];
        st.rc = match_recipe(st.fp);
    }
    if (!decode_fprog(rp->prog, rp->n_instr, n_ops, p.fp, slot_of))
        return fail(TADMA_ERR_UNSUPPORTED, "program step has no typed code");
    p.fp.acc = slot_of[rp->acc];
    p.rc = match_recipe(p.fp);
    p.out = (char*)o.data;
    p.out_rs = o.strides[0];
    if ((uintptr_t)o.data % 16 || (p.out_rs * dtype_size(o.dtype)) % (sizeof(float) == 4 && o.dtype != TADMA_F32 && es == 4 ? 8 : 16))
        return fail(TADMA_ERR_UNSUPPORTED, "out rows must be aligned for vector stores");
    // the typed kernels' fast-math rule (tadma_b200_eltwise)
    bool fast = rp->compute != TADMA_COMPUTE_F32_PRECISE && (o.dtype == TADMA_F16 || o.dtype == TADMA_BF16);
    for (int i = 0; i < rp->n_instr && fast; i++) {
        const int rd = rp->prog[i].round_dtype;
        if (!(rd < 0 || rd == TADMA_F32 || rd == TADMA_F16 || rd == TADMA_BF16)) fast = false;
    }
    p.fast = fast ? 1 : 0;
    cudaStream_t s = (cudaStream_t)stream;
    switch (ti) {
    case TADMA_F32: return launch_rp_i<float>(o.dtype, p, s);
    case TADMA_F16: return launch_rp_i<__half>(o.dtype, p, s);
    default: return launch_rp_i<__nv_bfloat16>(o.dtype, p, s);
    }
}
