// fill.cu - counter-based seeded generator (sm_100a).
//
// Element i of a tensor (global index g = offset + i) is a pure function of
// (seed, stream_id, g): the splitmix64 finaliser of a Weyl sequence keyed by
// (seed, stream_id).  Any shard therefore generates bit-identically on any
// GPU count, and the host oracle regenerates any element.  Floating values
// are built in double with explicitly rounded operations (no contraction)
// and rounded once to the element type.
//   UNIFORM: p0 + (p1 - p0) * (k * 2^-24),        k = top 24 bits of draw 0
//   NORMAL : p0 + p1 * z, z = sqrt(-2 ln u1) cos(2 pi t)  (Box-Muller, Box &
//            Muller 1958), u1 = (a + 1) 2^-53, t = b 2^-53 with a, b the top
//            53 bits of draws 0 and 1.  ln and cos are evaluated here from
//            their series with IEEE-rounded + - * / and sqrt only:
//              ln u = e ln2 + s * sum_j 2/(2j+1) s^2j, u = m 2^e,
//                     m in [sqrt(1/2), sqrt 2], s = (m - 1)/(m + 1);
//              cos 2 pi t folded to t in [0, 1/8] (cos(2pi(1-t)),
//                     -cos(2pi(1/2-t)), sin(2pi(1/4-t)); exact folds), then
//                     the Taylor series of cos or sin at x = 2 pi t.
//            No device math-library call is involved, so the host oracle
//            reproduces every value bit for bit; |z| reaches 8.6 (u1 = 2^-53).
//   INDEX  : floor(draw0 * n / 2^64)  (multiply-shift, bias < n / 2^64)
// The reference's randn (Operations.hpp:290-297) is host-only and seeded
// from std::random_device, so it cannot reproduce runs.
#include "common.cuh"
#include "layout.hpp"

namespace tadma_b200 {
namespace {

constexpr int THREADS = 256;
constexpr int LN_TERMS = 12;
constexpr int TRIG_TERMS = 9;

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t draw(uint64_t key, uint64_t g, uint64_t j) {
    return mix64(key + (4 * g + j + 1) * 0x9E3779B97F4A7C15ULL);
}

struct GenCoefs {
    double ln[LN_TERMS];   // 2 / (2j + 1)
    double cs[TRIG_TERMS]; // (-1)^k / (2k)!
    double sn[TRIG_TERMS]; // (-1)^k / (2k + 1)!
};

// Built on the host by exact-integer divisions (IEEE-rounded, the same on
// every machine).
GenCoefs make_coefs() {
    GenCoefs c{};
    for (int j = 0; j < LN_TERMS; j++) c.ln[j] = 2.0 / (double)(2 * j + 1);
    c.cs[0] = 1.0;
    c.sn[0] = 1.0;
    for (int k = 1; k < TRIG_TERMS; k++) {
        c.cs[k] = -c.cs[k - 1] / (double)((2 * k - 1) * (2 * k));
        c.sn[k] = -c.sn[k - 1] / (double)((2 * k) * (2 * k + 1));
    }
    return c;
}

__device__ __forceinline__ double gen_ln(const GenCoefs& c, double u) {  // u in (0, 1]
    const uint64_t bits = (uint64_t)__double_as_longlong(u);
    int e = (int)((bits >> 52) & 0x7ffu) - 1023;
    double m = __longlong_as_double((long long)((bits & 0xfffffffffffffULL) | 0x3ff0000000000000ULL));
    if (m > 0x1.6a09e667f3bcdp+0) {  // sqrt 2
        m = __dmul_rn(m, 0.5);
        e = e + 1;
    }
    const double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
    const double w = __dmul_rn(s, s);
    double p = c.ln[LN_TERMS - 1];
#pragma unroll
    for (int j = LN_TERMS - 2; j >= 0; j--) p = __dadd_rn(c.ln[j], __dmul_rn(w, p));
    return __dadd_rn(__dmul_rn((double)e, 0x1.62e42fefa39efp-1), __dmul_rn(s, p));  // ln 2
}

__device__ __forceinline__ double gen_cos_turns(const GenCoefs& c, double t) {  // t in [0, 1)
    bool neg = false, use_sin = false;
    if (t > 0.5) t = __dsub_rn(1.0, t);
    if (t > 0.25) {
        t = __dsub_rn(0.5, t);
        neg = true;
    }
    if (t > 0.125) {
        t = __dsub_rn(0.25, t);
        use_sin = true;
    }
    const double x = __dmul_rn(t, 0x1.921fb54442d18p+2);  // 2 pi
    const double y = __dmul_rn(x, x);
    const double* k = use_sin ? c.sn : c.cs;
    double p = k[TRIG_TERMS - 1];
#pragma unroll
    for (int j = TRIG_TERMS - 2; j >= 0; j--) p = __dadd_rn(k[j], __dmul_rn(y, p));
    if (use_sin) p = __dmul_rn(x, p);
    return neg ? -p : p;
}

struct FillParams {
    char* out;
    int32_t dtype, dist;
    double p0, p1, span;
    uint64_t key;
    uint64_t n_ids;
    int64_t offset, n;
    int32_t rank, contiguous;
    DivMod dm[TADMA_MAX_RANK];
    int64_t strides[TADMA_MAX_RANK];
    GenCoefs coefs;
};

__global__ void __launch_bounds__(THREADS) fill_kernel(const __grid_constant__ FillParams p) {
    pdl_begin();
    const int64_t stride = (int64_t)gridDim.x * THREADS;
    for (int64_t i = (int64_t)blockIdx.x * THREADS + threadIdx.x; i < p.n; i += stride) {
        int64_t off = i;
        if (!p.contiguous) {
            uint64_t e = (uint64_t)i;
            off = 0;
            for (int d = p.rank - 1; d >= 1; d--) {
                uint64_t q, r;
                p.dm[d].divmod(e, q, r);
                off += (int64_t)r * p.strides[d];
                e = q;
            }
            off += (int64_t)e * p.strides[0];
        }
        const uint64_t g = (uint64_t)(p.offset + i);
        if (p.dist == TADMA_DIST_INDEX) {
            const uint64_t id = __umul64hi(draw(p.key, g, 0), p.n_ids);
            store_from(p.out, p.dtype, off, (int64_t)id);
        } else if (p.dist == TADMA_DIST_UNIFORM) {
            const double u = __dmul_rn(__ull2double_rn(draw(p.key, g, 0) >> 40), 0x1p-24);
            store_from(p.out, p.dtype, off, __dadd_rn(p.p0, __dmul_rn(p.span, u)));
        } else {
            const double u1 = __dmul_rn(__ull2double_rn((draw(p.key, g, 0) >> 11) + 1), 0x1p-53);  // (0, 1]
            const double t = __dmul_rn(__ull2double_rn(draw(p.key, g, 1) >> 11), 0x1p-53);        // [0, 1)
            const double r = __dsqrt_rn(__dmul_rn(-2.0, gen_ln(p.coefs, u1)));
            const double z = __dmul_rn(r, gen_cos_turns(p.coefs, t));
            store_from(p.out, p.dtype, off, __dadd_rn(p.p0, __dmul_rn(p.p1, z)));
        }
    }
}

}  // namespace
}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_fill(const tadma_tensor* out, int32_t dist, double p0, double p1, uint64_t seed,
                               uint64_t stream_id, int64_t offset, void* stream) {
    std::string err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (dist < TADMA_DIST_UNIFORM || dist > TADMA_DIST_INDEX) return fail(TADMA_ERR_INVALID, "unknown distribution");
    if (dist == TADMA_DIST_INDEX && (dtype_is_float(out->dtype) || !(p1 >= 1.0)))
        return fail(TADMA_ERR_INVALID, "INDEX fills an integer tensor with n = p1 >= 1");
    if (dist != TADMA_DIST_INDEX && !dtype_is_float(out->dtype))
        return fail(TADMA_ERR_INVALID, "UNIFORM / NORMAL fill float tensors");
    if (offset < 0) return fail(TADMA_ERR_INVALID, "negative offset");
    const int64_t n = numel(out);
    if (n == 0) return TADMA_OK;
    FillParams p{};
    p.out = (char*)out->data;
    p.dtype = out->dtype;
    p.dist = dist;
    p.p0 = p0;
    p.p1 = p1;
    p.span = p1 - p0;
    p.key = mix64(seed ^ mix64(stream_id + 0x632BE59BD9B4E019ULL));
    p.n_ids = dist == TADMA_DIST_INDEX ? (uint64_t)p1 : 0;
    p.offset = offset;
    p.n = n;
    p.coefs = make_coefs();
    p.rank = out->rank > 0 ? out->rank : 1;
    // contiguous row-major?
    int64_t expect = 1;
    p.contiguous = 1;
    for (int d = out->rank - 1; d >= 0; d--) {
        if (out->dims[d] != 1 && out->strides[d] != expect) p.contiguous = 0;
        expect *= out->dims[d];
    }
    if (out->rank == 0) {
        p.dm[0] = DivMod(1);
        p.strides[0] = 0;
    }
    for (int d = 0; d < out->rank; d++) {
        p.dm[d] = DivMod((uint64_t)out->dims[d]);
        p.strides[d] = out->strides[d];
    }
    int64_t want = (n + THREADS - 1) / THREADS;
    int64_t cap = (int64_t)sm_count() * 8;
    int grid = (int)(want < cap ? want : cap);
    (void)launch_pdl(fill_kernel, dim3(grid), dim3(THREADS), 0, (cudaStream_t)stream, p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TADMA_OK : cuda_fail(e, "tadma_b200_fill launch");
}
