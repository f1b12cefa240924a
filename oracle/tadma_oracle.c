/*
 * tadma_oracle.c - CPU restatement of TADMA's element-wise / broadcast /
 * reduction / gather semantics.  TEST INFRASTRUCTURE ONLY (see header).
 *
 * PARITY UNPINNED: the reference cannot be compiled here and has no tests;
 * every function below cites the reference lines it restates (paths relative
 * to the OgnianM/TADMA project root) and is pinned by tests/golden KATs.
 *
 * Compile with -ffp-contract=off: float expressions must round after every
 * operation, exactly like the reference's one-op-per-node float arithmetic.
 */
#include "tadma_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ----------------------------------------------------------- conversions -- */

uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                  /* below 2^-14: subnormal half */
        float v;
        memcpy(&v, &ax, 4);
        uint32_t m = (uint32_t)nearbyintf(v * 16777216.0f); /* exact scaling, RNE */
        return (uint16_t)(sign | m);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t mant = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, bits;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e - 15 + 127) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t or_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7fffu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

float or_bf16_to_f32(uint16_t h) {
    uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}


static int is_float_dt(int32_t dt) {
    return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16 || dt == TADMA_F64;
}

/* float -> int64: truncate toward zero, saturate, NaN -> 0 (the sm_100
 * cvt.rzi.s64 rule the kernels use; C leaves it undefined). */
static int64_t f2i(double v) {
    if (v != v) return 0;
    if (v >= 9223372036854775807.0) return INT64_MAX;
    if (v <= -9223372036854775808.0) return INT64_MIN;
    return (int64_t)v;
}

/* Load element `off` (in elements) of a typed buffer as double. */
static double ld(const void* p, int32_t dt, int64_t off) {
    switch (dt) {
    case TADMA_F32: return ((const float*)p)[off];
    case TADMA_F16: return or_f16_to_f32(((const uint16_t*)p)[off]);
    case TADMA_BF16: return or_bf16_to_f32(((const uint16_t*)p)[off]);
    case TADMA_F64: return ((const double*)p)[off];
    case TADMA_I64: return (double)((const int64_t*)p)[off];
    case TADMA_I32: return ((const int32_t*)p)[off];
    case TADMA_U8: return ((const uint8_t*)p)[off];
    case TADMA_BOOL: return ((const uint8_t*)p)[off] != 0;
    case TADMA_I8: return ((const int8_t*)p)[off];
    }
    return 0;
}

static int64_t ldi(const void* p, int32_t dt, int64_t off) {
    switch (dt) {
    case TADMA_I64: return ((const int64_t*)p)[off];
    case TADMA_I32: return ((const int32_t*)p)[off];
    case TADMA_U8: return ((const uint8_t*)p)[off];
    case TADMA_BOOL: return ((const uint8_t*)p)[off] != 0;
    case TADMA_I8: return ((const int8_t*)p)[off];
    default: return f2i(ld(p, dt, off));
    }
}

/* Double -> fp16 / bf16 with ONE round-to-nearest-even step (no detour
 * through fp32, which could round twice).  The value is scaled by a power of
 * two (exact) so that the target's unit in the last place becomes 1, rounded
 * with nearbyint (the default rounding mode is nearest-even) and the bits are
 * rebuilt; the significand carry into the next binade and the subnormal range
 * fall out of the same formula.  NaN keeps the bits of the fp32 path. */
static uint16_t f64_to_16(double v, int man_bits, int emin, int bias, double inf_at, uint16_t inf_bits,
                          uint16_t (*nan_path)(float)) {
    uint64_t x;
    memcpy(&x, &v, 8);
    uint16_t sign = (uint16_t)((x >> 48) & 0x8000u);
    double a = fabs(v);
    if (v != v) return nan_path((float)v);
    if (a >= inf_at) return (uint16_t)(sign | inf_bits);
    if (a == 0.0) return sign;
    int e;
    (void)frexp(a, &e); /* a in [2^(e-1), 2^e) */
    int E = e - 1 < emin ? emin : e - 1;
    double m = nearbyint(ldexp(a, man_bits - E));
    return (uint16_t)(sign | (uint32_t)(((int64_t)(E + bias) << man_bits) + (int64_t)m - ((int64_t)1 << man_bits)));
}

uint16_t or_f64_to_f16(double v) {
    /* >= 65520 rounds to inf; normal exponents from -14, 10 stored bits */
    return f64_to_16(v, 10, -14, 15, 65520.0, 0x7c00u, or_f32_to_f16);
}

uint16_t or_f64_to_bf16(double v) {
    /* >= (2 - 2^-8) * 2^127 rounds to inf; normal exponents from -126, 7 stored bits */
    return f64_to_16(v, 7, -126, 127, ldexp(2.0 - ldexp(1.0, -8), 127), 0x7f80u, or_f32_to_bf16);
}

/* int64 -> bf16 in one rounding: below 2^53 the double is exact; above, the
 * 8 significant bits are rounded on the integer (ties to even). */
static uint16_t i64_to_bf16(int64_t v) {
    if (v > -(1LL << 53) && v < (1LL << 53)) return or_f64_to_bf16((double)v);
    uint64_t a = v < 0 ? 0 - (uint64_t)v : (uint64_t)v;
    int p = 63 - __builtin_clzll(a), sh = p - 7;
    uint64_t q = a >> sh, rem = a & ((1ULL << sh) - 1), half = 1ULL << (sh - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    double r = ldexp((double)q, sh); /* exact: q <= 256 */
    return or_f64_to_bf16(v < 0 ? -r : r);
}

/* Store a double: one rounding to the element type (fp32, fp16 and bf16 are
 * each rounded from the double; a double that holds an fp32 value gives the
 * same bits as rounding that fp32 value), integers truncate/saturate. */
static void st(void* p, int32_t dt, int64_t off, double v) {
    switch (dt) {
    case TADMA_F32: ((float*)p)[off] = (float)v; break;
    case TADMA_F16: ((uint16_t*)p)[off] = or_f64_to_f16(v); break;
    case TADMA_BF16: ((uint16_t*)p)[off] = or_f64_to_bf16(v); break;
    case TADMA_F64: ((double*)p)[off] = v; break;
    case TADMA_I64: ((int64_t*)p)[off] = f2i(v); break;
    case TADMA_I32: ((int32_t*)p)[off] = (int32_t)f2i(v); break;
    case TADMA_U8: ((uint8_t*)p)[off] = (uint8_t)f2i(v); break;
    case TADMA_BOOL: ((uint8_t*)p)[off] = v != 0; break;
    case TADMA_I8: ((int8_t*)p)[off] = (int8_t)f2i(v); break;
    }
}

static void sti(void* p, int32_t dt, int64_t off, int64_t v) {
    switch (dt) {
    case TADMA_I64: ((int64_t*)p)[off] = v; break;
    case TADMA_I32: ((int32_t*)p)[off] = (int32_t)v; break;
    case TADMA_U8: ((uint8_t*)p)[off] = (uint8_t)v; break;
    case TADMA_BOOL: ((uint8_t*)p)[off] = v != 0; break;
    case TADMA_I8: ((int8_t*)p)[off] = (int8_t)v; break;
    case TADMA_F32: ((float*)p)[off] = (float)v; break; /* one rounding (cvtsi2ss) */
    case TADMA_BF16: ((uint16_t*)p)[off] = i64_to_bf16(v); break;
    default: st(p, dt, off, (double)v); break; /* f16: |v| >= 2^53 is inf either way */
    }
}

/* Round an int64 to what a tensor of dtype `dt` would hold, read back as int64. */
static int64_t round_to_i(int64_t v, int32_t dt) {
    switch (dt) {
    case TADMA_F32: return f2i((double)(float)v);
    case TADMA_F16: return f2i(or_f16_to_f32(or_f64_to_f16((double)v)));
    case TADMA_BF16: return f2i(or_bf16_to_f32(i64_to_bf16(v)));
    case TADMA_F64: return f2i((double)v);
    case TADMA_I32: return (int32_t)v;
    case TADMA_U8: return (uint8_t)v;
    case TADMA_BOOL: return v != 0;
    case TADMA_I8: return (int8_t)v;
    }
    return v;
}

/* Round a double to what a tensor of dtype `dt` would hold. */
static double round_to(double v, int32_t dt) {
    switch (dt) {
    case TADMA_F32: return (float)v;
    case TADMA_F16: return or_f16_to_f32(or_f64_to_f16(v));
    case TADMA_BF16: return or_bf16_to_f32(or_f64_to_bf16(v));
    case TADMA_F64: return v;
    case TADMA_I64: return (double)f2i(v);
    case TADMA_I32: return (double)(int32_t)f2i(v);
    case TADMA_U8: return (double)(uint8_t)f2i(v);
    case TADMA_BOOL: return v != 0;
    case TADMA_I8: return (double)(int8_t)f2i(v);
    }
    return v;
}

/* ------------------------------------------------------ seeded generator -- */

uint64_t or_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static uint64_t gen_key(uint64_t seed, uint64_t stream_id) {
    return or_mix64(seed ^ or_mix64(stream_id + 0x632BE59BD9B4E019ULL));
}

static uint64_t gen_draw(uint64_t key, uint64_t idx, uint64_t j) {
    return or_mix64(key + (4 * idx + j + 1) * 0x9E3779B97F4A7C15ULL);
}

/* N(0, 1) by Box-Muller (G. E. P. Box and M. E. Muller, Ann. Math. Statist.
 * 29(2), 1958): z = sqrt(-2 ln u1) cos(2 pi t), one value per element from
 * its own two 53-bit uniforms.  ln and cos are evaluated here from their
 * series with IEEE-rounded +, -, *, / and sqrt only (no libm call), in the
 * same operation order as tadma_b200_fill, so host and device agree bit for
 * bit:
 *   ln u = e ln2 + 2 atanh(s) = e ln2 + s * sum_j 2/(2j+1) s^(2j),
 *          u = m 2^e, m in [sqrt(1/2), sqrt 2], s = (m - 1) / (m + 1);
 *   cos 2 pi t for t in turns, folded to [0, 1/8] by cos(2pi t) = cos(2pi(1-t)),
 *          = -cos(2pi(1/2-t)), = sin(2pi(1/4-t)) (each fold exact), then the
 *          Taylor series of cos or sin at x = 2 pi t <= pi/4.
 * The coefficients are built once by exact-integer divisions (gen_coefs). */
#define GEN_LN_TERMS 12
#define GEN_TRIG_TERMS 9
typedef struct {
    double ln[GEN_LN_TERMS];  /* 2 / (2j + 1) */
    double cs[GEN_TRIG_TERMS]; /* (-1)^k / (2k)! */
    double sn[GEN_TRIG_TERMS]; /* (-1)^k / (2k + 1)! */
} gen_coefs;

static void gen_coefs_init(gen_coefs* c) {
    for (int j = 0; j < GEN_LN_TERMS; j++) c->ln[j] = 2.0 / (double)(2 * j + 1);
    c->cs[0] = 1.0;
    c->sn[0] = 1.0;
    for (int k = 1; k < GEN_TRIG_TERMS; k++) {
        c->cs[k] = -c->cs[k - 1] / (double)((2 * k - 1) * (2 * k));
        c->sn[k] = -c->sn[k - 1] / (double)((2 * k) * (2 * k + 1));
    }
}

static double gen_ln(const gen_coefs* c, double u) { /* u in (0, 1] */
    uint64_t bits;
    memcpy(&bits, &u, 8);
    int e = (int)((bits >> 52) & 0x7ffu) - 1023;
    uint64_t mb = (bits & 0xfffffffffffffULL) | 0x3ff0000000000000ULL;
    double m;
    memcpy(&m, &mb, 8);
    if (m > 0x1.6a09e667f3bcdp+0) { /* sqrt 2 */
        m = m * 0.5;
        e = e + 1;
    }
    double s = (m - 1.0) / (m + 1.0);
    double w = s * s;
    double p = c->ln[GEN_LN_TERMS - 1];
    for (int j = GEN_LN_TERMS - 2; j >= 0; j--) p = c->ln[j] + w * p;
    return (double)e * 0x1.62e42fefa39efp-1 + s * p; /* ln 2 */
}

static double gen_cos_turns(const gen_coefs* c, double t) { /* t in [0, 1) */
    int neg = 0, use_sin = 0;
    if (t > 0.5) t = 1.0 - t;
    if (t > 0.25) {
        t = 0.5 - t;
        neg = 1;
    }
    if (t > 0.125) {
        t = 0.25 - t;
        use_sin = 1;
    }
    double x = t * 0x1.921fb54442d18p+2; /* 2 pi */
    double y = x * x;
    const double* k = use_sin ? c->sn : c->cs;
    double p = k[GEN_TRIG_TERMS - 1];
    for (int j = GEN_TRIG_TERMS - 2; j >= 0; j--) p = k[j] + y * p;
    if (use_sin) p = x * p;
    return neg ? -p : p;
}

static double gen_normal(const gen_coefs* c, uint64_t key, uint64_t g) {
    double u1 = (double)((gen_draw(key, g, 0) >> 11) + 1) * 0x1p-53; /* (0, 1] */
    double t = (double)(gen_draw(key, g, 1) >> 11) * 0x1p-53;        /* [0, 1) */
    double r = sqrt(-2.0 * gen_ln(c, u1));
    return r * gen_cos_turns(c, t);
}

double or_gen_normal(uint64_t seed, uint64_t stream_id, uint64_t g) {
    gen_coefs c;
    gen_coefs_init(&c);
    return gen_normal(&c, gen_key(seed, stream_id), g);
}

int or_fill(const tadma_tensor* out, int32_t dist, double p0, double p1, uint64_t seed,
            uint64_t stream_id, int64_t offset) {
    int64_t n = 1;
    for (int d = 0; d < out->rank; d++) n *= out->dims[d];
    uint64_t key = gen_key(seed, stream_id);
    double span = p1 - p0;
    gen_coefs coefs;
    gen_coefs_init(&coefs);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int64_t idx[TADMA_MAX_RANK], off = 0;
        or_map_to_shape(out->dims, out->rank, i, idx);
        for (int d = 0; d < out->rank; d++) off += idx[d] * out->strides[d];
        uint64_t g = (uint64_t)(offset + i);
        if (dist == TADMA_DIST_INDEX) {
            uint64_t h = gen_draw(key, g, 0);
            uint64_t id = (uint64_t)(((unsigned __int128)h * (uint64_t)p1) >> 64);
            sti(out->data, out->dtype, off, (int64_t)id);
        } else if (dist == TADMA_DIST_UNIFORM) {
            double u = (double)(gen_draw(key, g, 0) >> 40) * 0x1p-24;
            st(out->data, out->dtype, off, p0 + span * u);
        } else {
            st(out->data, out->dtype, off, p0 + p1 * gen_normal(&coefs, key, g));
        }
    }
    return TADMA_OK;
}

/* ---------------------------------------------------------- index helpers -- */

/* Utils.hpp:9-17: the last dimension is peeled first (constexpr_rfor). */
void or_map_to_shape(const int64_t* dims, int32_t rank, int64_t index, int64_t* out_idx) {
    for (int d = rank - 1; d >= 0; d--) {
        out_idx[d] = index % dims[d];
        index /= dims[d];
    }
}

static int64_t numel(const tadma_tensor* t) {
    int64_t n = 1;
    for (int d = 0; d < t->rank; d++) n *= t->dims[d];
    return n;
}

static int64_t offset_of(const tadma_tensor* t, const int64_t* idx) {
    int64_t off = 0;
    for (int d = 0; d < t->rank; d++) off += idx[d] * t->strides[d];
    return off;
}

/* ----------------------------------------------------------- element-wise -- */

static int is_transcendental(int32_t op) {
    return (op >= TADMA_OP_EXP && op <= TADMA_OP_GELU) && op != TADMA_OP_RELU;
}

/* Operations.hpp:160-164 defines tanh(x) = (e^x - e^-x) / (e^x + e^-x).  That
 * equals expm1(2x) / (expm1(2x) + 2), which is evaluated here instead: it has
 * no cancellation near 0 and no inf/inf (NaN) for |x| > ~355, where the
 * reference expression breaks down (documented deviation). */
static double tanh_ref(double x) {
    if (x > 20.0) return 1.0; /* 1 - 2e^-2x rounds to 1 in double */
    if (x < -20.0) return -1.0;
    double e = expm1(2.0 * x);
    return e / (e + 2.0);
}

/* Operations.hpp:181: 0.5 * x * (1 + tanh(0.7978845608 * (x + 0.044715 * x^3))).
 * 0.5 (1 + tanh(u)) == 1 / (1 + e^-2u), so gelu = x / (1 + exp(-2u)): the same
 * function without the catastrophic cancellation of 1 + tanh(u) for x < -3
 * (the reference expression returns exactly -0 below x ~ -9 even in double). */
static double gelu_ref(double x) {
    double u = 0.7978845608 * (x + 0.044715 * x * x * x);
    return x / (1.0 + exp(-2.0 * u));
}

/* unary op in double (transcendentals) */
static double unary_d(int32_t op, double x) {
    switch (op) {
    case TADMA_OP_COPY: return x;
    case TADMA_OP_NEG: return -x;
    case TADMA_OP_ABS: return fabs(x);
    case TADMA_OP_EXP: return exp(x);
    case TADMA_OP_LOG: return log(x);
    case TADMA_OP_SQRT: return sqrt(x);
    case TADMA_OP_SIN: return sin(x);
    case TADMA_OP_COS: return cos(x);
    case TADMA_OP_TAN: return tan(x);
    case TADMA_OP_ASIN: return asin(x);
    case TADMA_OP_ACOS: return acos(x);
    case TADMA_OP_ATAN: return atan(x);
    case TADMA_OP_ASINH: return asinh(x);
    case TADMA_OP_ACOSH: return acosh(x);
    case TADMA_OP_ATANH: return atanh(x);
    case TADMA_OP_ERF: return erf(x);
    case TADMA_OP_RELU: return x > 0 ? x : 0; /* Operations.hpp:178 */
    case TADMA_OP_SIGMOID: return 1 / (1 + exp(-x)); /* Operations.hpp:179 */
    case TADMA_OP_TANH: return tanh_ref(x);
    case TADMA_OP_GELU: return gelu_ref(x);
    case TADMA_OP_NOT: return x == 0;
    }
    return NAN;
}

static int resolve_compute(const tadma_tensor* out, const tadma_tensor* ins, int32_t n_ins,
                           const tadma_instr* prog, int32_t n_instr, int32_t compute) {
    if (compute == TADMA_COMPUTE_F32_PRECISE) return TADMA_COMPUTE_F32; /* the oracle has no fast-math bodies */
    if (compute != TADMA_COMPUTE_AUTO) return compute;
    int all_int = !is_float_dt(out->dtype), any_wide = out->dtype == TADMA_F64 || out->dtype == TADMA_I64;
    for (int k = 0; k < n_ins; k++) {
        if (is_float_dt(ins[k].dtype)) all_int = 0;
        if (ins[k].dtype == TADMA_F64 || ins[k].dtype == TADMA_I64) any_wide = 1;
    }
    for (int i = 0; i < n_instr; i++) {
        if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW) all_int = 0;
        if ((prog[i].b == TADMA_SRC_IMM || prog[i].c == TADMA_SRC_IMM) && prog[i].imm != floor(prog[i].imm)) all_int = 0;
    }
    if (all_int) return TADMA_COMPUTE_I64;
    return any_wide ? TADMA_COMPUTE_F64 : TADMA_COMPUTE_F32;
}

/* Binary / ternary op, float or double compute (no contraction: -ffp-contract=off). */
#define BIN_BODY(T)                                                                   \
    switch (op) {                                                                     \
    case TADMA_OP_ADD: return a + b;                                                  \
    case TADMA_OP_SUB: return a - b;                                                  \
    case TADMA_OP_MUL: return a * b;                                                  \
    case TADMA_OP_DIV: return a / b;                                                  \
    case TADMA_OP_RSUB: return b - a;                                                 \
    case TADMA_OP_RDIV: return b / a;                                                 \
    case TADMA_OP_MAX: return (a < b) ? b : a; /* std::max(a, b) */                  \
    case TADMA_OP_MIN: return (b < a) ? b : a; /* std::min(a, b) */                  \
    case TADMA_OP_EQ: return a == b;                                                  \
    case TADMA_OP_NE: return a != b;                                                  \
    case TADMA_OP_LT: return a < b;                                                   \
    case TADMA_OP_GT: return a > b;                                                   \
    case TADMA_OP_LE: return a <= b;                                                  \
    case TADMA_OP_GE: return a >= b;                                                  \
    case TADMA_OP_AND: case TADMA_OP_LAND: return (a != 0) && (b != 0);               \
    case TADMA_OP_OR: case TADMA_OP_LOR: return (a != 0) || (b != 0);                 \
    case TADMA_OP_XOR: return (a != 0) != (b != 0);                                   \
    case TADMA_OP_WHERE: return (a != 0) ? b : c;                                     \
    }                                                                                 \
    return (T)NAN;

static float bin_f(int32_t op, float a, float b, float c) { BIN_BODY(float) }
static double bin_d(int32_t op, double a, double b, double c) { BIN_BODY(double) }

static int64_t bin_i(int32_t op, int64_t a, int64_t b, int64_t c) {
    switch (op) {
    case TADMA_OP_ADD: return (int64_t)((uint64_t)a + (uint64_t)b);
    case TADMA_OP_SUB: return (int64_t)((uint64_t)a - (uint64_t)b);
    case TADMA_OP_MUL: return (int64_t)((uint64_t)a * (uint64_t)b);
    case TADMA_OP_DIV: return b == 0 ? 0 : (b == -1 ? (int64_t)(0 - (uint64_t)a) : a / b);
    case TADMA_OP_RSUB: return (int64_t)((uint64_t)b - (uint64_t)a);
    case TADMA_OP_RDIV: return a == 0 ? 0 : (a == -1 ? (int64_t)(0 - (uint64_t)b) : b / a);
    case TADMA_OP_MAX: return (a < b) ? b : a;
    case TADMA_OP_MIN: return (b < a) ? b : a;
    case TADMA_OP_EQ: return a == b;
    case TADMA_OP_NE: return a != b;
    case TADMA_OP_LT: return a < b;
    case TADMA_OP_GT: return a > b;
    case TADMA_OP_LE: return a <= b;
    case TADMA_OP_GE: return a >= b;
    case TADMA_OP_AND: return a & b;
    case TADMA_OP_OR: return a | b;
    case TADMA_OP_XOR: return a ^ b;
    case TADMA_OP_LAND: return (a != 0) && (b != 0);
    case TADMA_OP_LOR: return (a != 0) || (b != 0);
    case TADMA_OP_WHERE: return (a != 0) ? b : c;
    case TADMA_OP_COPY: return a;
    case TADMA_OP_NEG: return (int64_t)(0 - (uint64_t)a);
    case TADMA_OP_ABS: return a < 0 ? (int64_t)(0 - (uint64_t)a) : a;
    case TADMA_OP_RELU: return a > 0 ? a : 0;
    case TADMA_OP_NOT: return a == 0;
    }
    return 0;
}

static int op_is_unary(int32_t op) { return op < 32; }

/*
 * Chain semantics (the fused form of Kernels.hpp:16-53 + Node.hpp:189-224):
 * acc = ins[0]; acc = op_i(acc, b_i, c_i) with an optional rounding to
 * round_dtype after each op; out = acc.  Iteration order is MapToShape order
 * over out's dims (Utils.hpp:9-17), which for element-wise maps is immaterial.
 */
int or_eltwise(const tadma_tensor* out, const tadma_tensor* ins, int32_t n_ins,
               const tadma_instr* prog, int32_t n_instr, int32_t compute) {
    if (n_instr < 0 || n_instr > TADMA_MAX_INSTR || n_ins < 0 || n_ins > TADMA_MAX_INPUTS) return TADMA_ERR_INVALID;
    int cm = resolve_compute(out, ins, n_ins, prog, n_instr, compute);
    int64_t n = numel(out);
#pragma omp parallel for schedule(static)
    for (int64_t e = 0; e < n; e++) {
        int64_t idx[TADMA_MAX_RANK];
        or_map_to_shape(out->dims, out->rank, e, idx);
        double vin[TADMA_MAX_INPUTS];
        int64_t iin[TADMA_MAX_INPUTS];
        for (int k = 0; k < n_ins; k++) {
            int64_t off = offset_of(&ins[k], idx);
            if (cm == TADMA_COMPUTE_I64) iin[k] = ldi(ins[k].data, ins[k].dtype, off);
            else vin[k] = ld(ins[k].data, ins[k].dtype, off);
        }
        if (cm == TADMA_COMPUTE_I64) {
            int64_t acc = n_ins > 0 ? iin[0] : 0;
            for (int i = 0; i < n_instr; i++) {
                const tadma_instr* I = &prog[i];
                int64_t b = I->b >= 0 ? iin[I->b] : (int64_t)I->imm;
                int64_t c = I->c >= 0 ? iin[I->c] : (int64_t)I->imm;
                if (op_is_unary(I->op)) acc = (I->op == TADMA_OP_COPY && I->b == TADMA_SRC_IMM) ? b : bin_i(I->op, acc, 0, 0);
                else acc = bin_i(I->op, acc, b, c);
                if (I->round_dtype >= 0) acc = round_to_i(acc, I->round_dtype);
            }
            sti(out->data, out->dtype, offset_of(out, idx), acc);
        } else if (cm == TADMA_COMPUTE_F32) {
            float fin[TADMA_MAX_INPUTS];
            for (int k = 0; k < n_ins; k++) /* an int64 input rounds to fp32 once, as load_as<float> does */
                fin[k] = ins[k].dtype == TADMA_I64 ? (float)((const int64_t*)ins[k].data)[offset_of(&ins[k], idx)] : (float)vin[k];
            float acc = n_ins > 0 ? fin[0] : 0.0f;
            for (int i = 0; i < n_instr; i++) {
                const tadma_instr* I = &prog[i];
                float b = I->b >= 0 ? fin[I->b] : (float)I->imm;
                float c = I->c >= 0 ? fin[I->c] : (float)I->imm;
                if (I->op == TADMA_OP_COPY && I->b == TADMA_SRC_IMM) acc = b;
                else if (I->op == TADMA_OP_POW) acc = (b == 2.0f) ? acc * acc : (float)pow((double)acc, (double)b);
                else if (op_is_unary(I->op)) {
                    if (I->op == TADMA_OP_NEG) acc = -acc;
                    else if (I->op == TADMA_OP_ABS) acc = fabsf(acc);
                    else if (I->op == TADMA_OP_RELU) acc = acc > 0 ? acc : 0.0f;
                    else if (I->op == TADMA_OP_NOT) acc = acc == 0;
                    else acc = (float)unary_d(I->op, (double)acc);
                } else acc = bin_f(I->op, acc, b, c);
                if (I->round_dtype >= 0) acc = (float)round_to((double)acc, I->round_dtype);
            }
            st(out->data, out->dtype, offset_of(out, idx), (double)acc);
        } else {
            double acc = n_ins > 0 ? vin[0] : 0.0;
            for (int i = 0; i < n_instr; i++) {
                const tadma_instr* I = &prog[i];
                double b = I->b >= 0 ? vin[I->b] : I->imm;
                double c = I->c >= 0 ? vin[I->c] : I->imm;
                if (I->op == TADMA_OP_COPY && I->b == TADMA_SRC_IMM) acc = b;
                else if (I->op == TADMA_OP_POW) acc = (b == 2.0) ? acc * acc : pow(acc, b);
                else if (op_is_unary(I->op)) acc = unary_d(I->op, acc);
                else acc = bin_d(I->op, acc, b, c);
                if (I->round_dtype >= 0) acc = round_to(acc, I->round_dtype);
            }
            st(out->data, out->dtype, offset_of(out, idx), acc);
        }
    }
    return TADMA_OK;
}

/* -------------------------------------------------------------- reduction -- */

static int norm_axis(int32_t axis, int32_t rank) {
    if (axis < 0) axis += rank;
    return (axis < 0 || axis >= rank) ? -1 : axis;
}

/*
 * ReduceNode / ReduceKernel (kernels/Reduce.hpp:10-71) + Tensor::sum/min/max/
 * mean (Tensor.hpp:436-448).  Accumulation is fp64 for float inputs and
 * int64 for integer inputs (the reference's decltype(a + b)); MEAN of an
 * integer tensor divides as integers (x / Dim(D), Tensor.hpp:448).  MAX/MIN
 * propagate NaN.  ARGMAX/ARGMIN return the first extreme index, NaN counting
 * as the extreme (numpy semantics).  pre_op is applied in double and rounded
 * to fp32, the dtype the reference's materialised pre-op tensor would have.
 */
int or_reduce(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op, const tadma_tensor* out) {
    int ax = norm_axis(axis, in->rank);
    if (ax < 0) return TADMA_ERR_INVALID;
    int keep = out->rank == in->rank;
    int64_t R = in->dims[ax];
    /* An empty reduction has an identity only for the sums; the C ABI
     * rejects the others (there is no first element to return). */
    if (R == 0 && op != TADMA_REDUCE_SUM && op != TADMA_REDUCE_SUMSQ) return TADMA_ERR_INVALID;
    int64_t n_out = numel(in) / (R ? R : 1);
    if (R == 0) n_out = numel(out);
    int64_t odims[TADMA_MAX_RANK];
    int orank = 0;
    for (int d = 0; d < in->rank; d++)
        if (d != ax) odims[orank++] = in->dims[d];
    int isint = !is_float_dt(in->dtype);
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < n_out; o++) {
        int64_t oidx[TADMA_MAX_RANK], iidx[TADMA_MAX_RANK], outidx[TADMA_MAX_RANK];
        or_map_to_shape(odims, orank, o, oidx);
        for (int d = 0, k = 0; d < in->rank; d++) iidx[d] = (d == ax) ? 0 : oidx[k++];
        for (int d = 0, k = 0; d < out->rank; d++) outidx[d] = keep ? iidx[d] : oidx[k++];
        int64_t ooff = offset_of(out, outidx);
        int64_t base = offset_of(in, iidx);
        if (op == TADMA_REDUCE_ARGMAX || op == TADMA_REDUCE_ARGMIN) {
            int64_t best = 0;
            double bv = 0;
            for (int64_t r = 0; r < R; r++) {
                double v = ld(in->data, in->dtype, base + r * in->strides[ax]);
                if (pre_op != TADMA_OP_COPY) v = (float)unary_d(pre_op, v);
                if (r == 0) { bv = v; best = 0; continue; }
                if (bv != bv) break; /* first NaN wins */
                int better = (op == TADMA_REDUCE_ARGMAX) ? (v > bv) : (v < bv);
                if (v != v || better) { bv = v; best = r; }
            }
            sti(out->data, out->dtype, ooff, best);
            continue;
        }
        if (isint && pre_op == TADMA_OP_COPY && op != TADMA_REDUCE_RMS) {
            int64_t acc = 0;
            for (int64_t r = 0; r < R; r++) {
                int64_t v = ldi(in->data, in->dtype, base + r * in->strides[ax]);
                if (op == TADMA_REDUCE_SUMSQ) v = v * v;
                if (r == 0 && (op == TADMA_REDUCE_MAX || op == TADMA_REDUCE_MIN)) acc = v;
                else if (op == TADMA_REDUCE_MAX) acc = v > acc ? v : acc;
                else if (op == TADMA_REDUCE_MIN) acc = v < acc ? v : acc;
                else acc += v;
            }
            if (op == TADMA_REDUCE_MEAN) acc = R ? acc / R : 0;
            sti(out->data, out->dtype, ooff, acc);
            continue;
        }
        double acc = 0;
        for (int64_t r = 0; r < R; r++) {
            double v = ld(in->data, in->dtype, base + r * in->strides[ax]);
            if (pre_op != TADMA_OP_COPY) v = (float)unary_d(pre_op, v);
            if (op == TADMA_REDUCE_SUMSQ || op == TADMA_REDUCE_RMS) v = v * v;
            if (r == 0 && (op == TADMA_REDUCE_MAX || op == TADMA_REDUCE_MIN)) acc = v;
            else if (op == TADMA_REDUCE_MAX) acc = (acc != acc || v != v) ? NAN : (v > acc ? v : acc);
            else if (op == TADMA_REDUCE_MIN) acc = (acc != acc || v != v) ? NAN : (v < acc ? v : acc);
            else acc += v;
        }
        if (op == TADMA_REDUCE_MEAN) acc = acc / (double)R;
        if (op == TADMA_REDUCE_RMS) acc = sqrt(acc / (double)R);
        st(out->data, out->dtype, ooff, acc);
    }
    return TADMA_OK;
}

/* ------------------------------------------------ fused reduce+broadcast -- */

/* Shared row walker: calls fn for every row along `ax`. */
typedef void (*row_fn)(const tadma_tensor* in, const tadma_tensor* out, int64_t ibase, int64_t obase,
                       int64_t istride, int64_t ostride, int64_t R, const void* ctx);

static int for_rows(const tadma_tensor* in, int32_t axis, const tadma_tensor* out, row_fn fn, const void* ctx) {
    int ax = norm_axis(axis, in->rank);
    if (ax < 0) return TADMA_ERR_INVALID;
    int64_t R = in->dims[ax];
    int64_t odims[TADMA_MAX_RANK];
    int orank = 0;
    for (int d = 0; d < in->rank; d++)
        if (d != ax) odims[orank++] = in->dims[d];
    int64_t nrows = R ? numel(in) / R : 0;
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < nrows; o++) {
        int64_t oidx[TADMA_MAX_RANK], iidx[TADMA_MAX_RANK];
        or_map_to_shape(odims, orank, o, oidx);
        for (int d = 0, k = 0; d < in->rank; d++) iidx[d] = (d == ax) ? 0 : oidx[k++];
        fn(in, out, offset_of(in, iidx), offset_of(out, iidx), in->strides[ax], out->strides[ax], R, ctx);
    }
    return TADMA_OK;
}

/* softmax (Operations.hpp:190-193): exp(x) / sum(exp(x)), restated with the
 * max subtracted (equal in exact arithmetic, no fp16 overflow), in double. */
static void softmax_row(const tadma_tensor* in, const tadma_tensor* out, int64_t ib, int64_t ob,
                        int64_t is, int64_t os, int64_t R, const void* ctx) {
    (void)ctx;
    double m = -INFINITY, s = 0;
    for (int64_t r = 0; r < R; r++) {
        double v = ld(in->data, in->dtype, ib + r * is);
        if (v > m || v != v) m = v;
    }
    for (int64_t r = 0; r < R; r++) s += exp(ld(in->data, in->dtype, ib + r * is) - m);
    double* tmp = (double*)malloc(sizeof(double) * (size_t)(R ? R : 1));
    for (int64_t r = 0; r < R; r++) tmp[r] = exp(ld(in->data, in->dtype, ib + r * is) - m) / s;
    for (int64_t r = 0; r < R; r++) st(out->data, out->dtype, ob + r * os, tmp[r]);
    free(tmp);
}

int or_softmax(const tadma_tensor* in, int32_t axis, const tadma_tensor* out) {
    return for_rows(in, axis, out, softmax_row, NULL);
}

typedef struct {
    const tadma_tensor *gamma, *beta;
    double eps;
    int32_t mode;
} ln_ctx;

/* mean_stddev + layer_norm (Operations.hpp:195-220): population std; the
 * reference adds eps to the std (TADMA_LN_TADMA), ONNX graphs add it to the
 * variance (TADMA_LN_ONNX).  Double math, one rounding to the output dtype. */
static void ln_row(const tadma_tensor* in, const tadma_tensor* out, int64_t ib, int64_t ob,
                   int64_t is, int64_t os, int64_t R, const void* vctx) {
    const ln_ctx* c = (const ln_ctx*)vctx;
    double mean = 0, var = 0;
    for (int64_t r = 0; r < R; r++) mean += ld(in->data, in->dtype, ib + r * is);
    mean /= (double)R;
    for (int64_t r = 0; r < R; r++) {
        double d = ld(in->data, in->dtype, ib + r * is) - mean;
        var += d * d;
    }
    var /= (double)R;
    double denom = c->mode == TADMA_LN_TADMA ? sqrt(var) + c->eps : sqrt(var + c->eps);
    double* tmp = (double*)malloc(sizeof(double) * (size_t)(R ? R : 1));
    for (int64_t r = 0; r < R; r++) {
        double g = (c->gamma && c->gamma->data) ? ld(c->gamma->data, c->gamma->dtype, r * c->gamma->strides[0]) : 1.0;
        double b = (c->beta && c->beta->data) ? ld(c->beta->data, c->beta->dtype, r * c->beta->strides[0]) : 0.0;
        tmp[r] = (ld(in->data, in->dtype, ib + r * is) - mean) / denom * g + b;
    }
    for (int64_t r = 0; r < R; r++) st(out->data, out->dtype, ob + r * os, tmp[r]);
    free(tmp);
}

int or_layer_norm(const tadma_tensor* in, int32_t axis, const tadma_tensor* gamma,
                  const tadma_tensor* beta, double eps, int32_t mode, const tadma_tensor* out) {
    ln_ctx c = {gamma, beta, eps, mode};
    return for_rows(in, axis, out, ln_row, &c);
}

/* rms_norm (Operations.hpp:222-233): x / sqrt(mean(x^2)) (+ eps, 0 = reference) */
static void rms_row(const tadma_tensor* in, const tadma_tensor* out, int64_t ib, int64_t ob,
                    int64_t is, int64_t os, int64_t R, const void* vctx) {
    double eps = *(const double*)vctx, ss = 0;
    for (int64_t r = 0; r < R; r++) {
        double v = ld(in->data, in->dtype, ib + r * is);
        ss += v * v;
    }
    double d = sqrt(ss / (double)R + eps);
    double* tmp = (double*)malloc(sizeof(double) * (size_t)(R ? R : 1));
    for (int64_t r = 0; r < R; r++) tmp[r] = ld(in->data, in->dtype, ib + r * is) / d;
    for (int64_t r = 0; r < R; r++) st(out->data, out->dtype, ob + r * os, tmp[r]);
    free(tmp);
}

int or_rms_norm(const tadma_tensor* in, int32_t axis, double eps, const tadma_tensor* out) {
    return for_rows(in, axis, out, rms_row, &eps);
}

/* ----------------------------------------------------------------- gather -- */

/*
 * ONNX Gather (Operations.hpp:244-262 states the intent; its rank-2-ids path
 * is broken, this restates the ONNX definition it links to):
 * out[a.., j.., b..] = table[a.., ids[j..], b..] (+ add[a.., j.., b..]).
 * Negative ids count from the end; ids outside [-n, n) give 0 (+ add) and
 * TADMA_ERR_INDEX.  Math in fp32: float(table) + float(add), one rounding.
 */
int or_gather(const tadma_tensor* table, int32_t axis, const tadma_tensor* ids,
              const tadma_tensor* add, const tadma_tensor* out) {
    int ax = norm_axis(axis, table->rank);
    if (ax < 0) return TADMA_ERR_INVALID;
    int64_t n = table->dims[ax];
    int64_t total = numel(out);
    int bad = 0;
    int has_add = add && add->data;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t e = 0; e < total; e++) {
        int64_t oidx[TADMA_MAX_RANK], tidx[TADMA_MAX_RANK], jidx[TADMA_MAX_RANK];
        or_map_to_shape(out->dims, out->rank, e, oidx);
        for (int d = 0; d < ids->rank; d++) jidx[d] = oidx[ax + d];
        int64_t id = ldi(ids->data, ids->dtype, offset_of(ids, jidx));
        if (id < 0) id += n;
        float v = 0.0f;
        if (id < 0 || id >= n) {
            bad = 1;
        } else {
            for (int d = 0; d < ax; d++) tidx[d] = oidx[d];
            tidx[ax] = id;
            for (int d = ax + 1; d < table->rank; d++) tidx[d] = oidx[d - 1 + ids->rank];
            v = (float)ld(table->data, table->dtype, offset_of(table, tidx));
        }
        if (has_add) v = v + (float)ld(add->data, add->dtype, offset_of(add, oidx));
        st(out->data, out->dtype, offset_of(out, oidx), (double)v);
    }
    return bad ? TADMA_ERR_INDEX : TADMA_OK;
}

/* ------------------------------------------- per-config straightforward loops -- */

/* Config 2, y = gelu(x * s + bias) as the reference evaluates it: x*s and
 * +bias are float nodes (bf16 promotes to float, Tensor.hpp:499-501,524),
 * gelu's lambda runs in double (0.5 is a double literal, Operations.hpp:181)
 * and its in-place store rounds to float; the bf16 output rounds that. */
void or_cfg2_gelu_affine_bf16(const uint16_t* x, const uint16_t* bias, float s, uint16_t* y,
                              int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t c = 0; c < cols; c++) {
            float t = or_bf16_to_f32(x[r * cols + c]) * s;
            t = t + or_bf16_to_f32(bias[c]);
            float g = (float)gelu_ref((double)t);
            y[r * cols + c] = or_f32_to_bf16(g);
        }
    }
}

void or_cfg3_sum_lastaxis_f32(const float* x, float* y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        double acc = 0;
        for (int64_t c = 0; c < cols; c++) acc += x[r * cols + c];
        y[r] = (float)acc;
    }
}

void or_cfg3_max_lastaxis_f32(const float* x, float* y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        float m = x[r * cols];
        for (int64_t c = 1; c < cols; c++) {
            float v = x[r * cols + c];
            if (m != m || v != v) m = NAN;
            else if (v > m) m = v;
        }
        y[r] = m;
    }
}

void or_cfg3_argmax_lastaxis_f32(const float* x, int64_t* y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        float m = x[r * cols];
        int64_t b = 0;
        for (int64_t c = 1; c < cols && m == m; c++) {
            float v = x[r * cols + c];
            if (v != v || v > m) { m = v; b = c; }
        }
        y[r] = b;
    }
}

void or_cfg3_mean_midaxis_f32(const float* x, float* y, int64_t outer, int64_t R, int64_t inner) {
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < outer; o++) {
        double* acc = (double*)calloc((size_t)inner, sizeof(double));
        for (int64_t r = 0; r < R; r++)
            for (int64_t i = 0; i < inner; i++) acc[i] += x[(o * R + r) * inner + i];
        for (int64_t i = 0; i < inner; i++) y[o * inner + i] = (float)(acc[i] / (double)R);
        free(acc);
    }
}

/* The reference's own fold order and accumulator type for a reduction over
 * rows (include/tadma/kernels/Reduce.hpp:10-55, ReduceNode :58-69): Threads =
 * min(1024, floor_pow2(R)); thread t folds elements t, t + Threads, ... in
 * increasing order; then a shared-memory tree halves the partials (partial t
 * += partial t + i for i = Threads / 2 .. 1).  The accumulator is decltype(a
 * + b) of the element type: fp32 for fp32, fp16 for fp16 (every fp16 add
 * rounds once to fp16, as __hadd does; the exact sum of two fp16 values fits
 * a double).  op: 0 sum, 1 max (std::max: a < b ? b : a, so a NaN survives
 * only where it lands in the accumulator), 2 mean (the sum divided by R in
 * the accumulator type, Tensor.hpp:448).  dtype TADMA_F32 or TADMA_F16;
 * R >= 1.  Returns 0, or -1 for an unsupported dtype / op. */
static double ref_acc_add(double a, double b, int32_t dt) {
    return dt == TADMA_F16 ? (double)or_f16_to_f32(or_f64_to_f16(a + b)) : (double)(float)((float)a + (float)b);
}
static double ref_acc_max(double a, double b) { return a < b ? b : a; }
int or_reduce_rows_reference_order(int32_t op, const void* x, int32_t dtype, int64_t rows, int64_t R, void* out) {
    if ((dtype != TADMA_F32 && dtype != TADMA_F16) || op < 0 || op > 2 || R < 1) return -1;
    int64_t th = 1;
    while (th * 2 <= R && th < 1024) th *= 2;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        double part[1024];
        for (int64_t t = 0; t < th; t++) {
            double v = ld(x, dtype, r * R + t);
            for (int64_t i = t + th; i < R; i += th) {
                double e = ld(x, dtype, r * R + i);
                v = op == 1 ? ref_acc_max(v, e) : ref_acc_add(v, e, dtype);
            }
            part[t] = v;
        }
        for (int64_t i = th / 2; i > 0; i /= 2)
            for (int64_t t = 0; t < i; t++)
                part[t] = op == 1 ? ref_acc_max(part[t], part[t + i]) : ref_acc_add(part[t], part[t + i], dtype);
        double v = part[0];
        if (op == 2) {
            v = dtype == TADMA_F16 ? (double)or_f16_to_f32(or_f64_to_f16(v / (double)or_f16_to_f32(or_f64_to_f16((double)R))))
                                   : (double)((float)v / (float)R);
        }
        st(out, dtype, r, v);
    }
    return 0;
}

void or_cfg4_layer_norm_f16(const uint16_t* x, const uint16_t* g, const uint16_t* b, double eps,
                            uint16_t* y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const uint16_t* xr = x + r * cols;
        double mean = 0, var = 0;
        for (int64_t c = 0; c < cols; c++) mean += or_f16_to_f32(xr[c]);
        mean /= (double)cols;
        for (int64_t c = 0; c < cols; c++) {
            double d = or_f16_to_f32(xr[c]) - mean;
            var += d * d;
        }
        double rs = 1.0 / sqrt(var / (double)cols + eps);
        for (int64_t c = 0; c < cols; c++)
            y[r * cols + c] = or_f32_to_f16((float)((or_f16_to_f32(xr[c]) - mean) * rs * or_f16_to_f32(g[c]) + or_f16_to_f32(b[c])));
    }
}

void or_cfg4_softmax_f16(const uint16_t* x, uint16_t* y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const uint16_t* xr = x + r * cols;
        double m = -INFINITY, s = 0;
        for (int64_t c = 0; c < cols; c++) {
            double v = or_f16_to_f32(xr[c]);
            if (v > m) m = v;
        }
        for (int64_t c = 0; c < cols; c++) s += exp(or_f16_to_f32(xr[c]) - m);
        double inv = 1.0 / s;
        for (int64_t c = 0; c < cols; c++) y[r * cols + c] = or_f32_to_f16((float)(exp(or_f16_to_f32(xr[c]) - m) * inv));
    }
}

void or_cfg5_gather_add(const uint16_t* table_f16, int64_t vocab, const int64_t* ids,
                        const uint16_t* pos_bf16, uint16_t* out_bf16, int64_t batch, int64_t seq,
                        int64_t dim) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < batch * seq; row++) {
        int64_t s = row % seq, id = ids[row];
        if (id < 0) id += vocab;
        const uint16_t* t = (id >= 0 && id < vocab) ? table_f16 + id * dim : NULL;
        const uint16_t* p = pos_bf16 + s * dim;
        uint16_t* o = out_bf16 + row * dim;
        for (int64_t d = 0; d < dim; d++) {
            float v = t ? or_f16_to_f32(t[d]) : 0.0f;
            o[d] = or_f32_to_bf16(v + or_bf16_to_f32(p[d]));
        }
    }
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
    omp_set_num_threads(n);
#else
    (void)n;
#endif
}
