// kdiv.cuh - correctly rounded fp32 division by a divisor that many
// dividends share (a row's standard deviation in a LayerNorm tail).
//
// The reciprocal y = RN(1/b) is taken once per divisor; each quotient then
// costs one multiply and four fused multiply-adds (Markstein, "Computation
// of elementary functions on the IBM RISC System/6000 processor", IBM J.
// Res. Dev. 34(1), 1990; the quotient theorem as stated in Muller et al.,
// "Handbook of Floating-Point Arithmetic", 2nd ed., 2018, section 4.7):
//
//   q0 = RN(a y)                   q0 = (a/b)(1 + e0), |e0| <= 2^-23 + 2^-48
//   q1 = RN(q0 + RN(a - b q0) y)   before rounding q1 is (a/b)(1 + e1) with
//                                  |e1| <= |e0| (2^-23 + 2^-48) < 2^-45, so
//                                  q1 is within one ulp of a/b (faithful)
//   q2 = RN(q1 + (a - b q1) y)     q1 faithful makes a - b q1 a float, which
//                                  the fused multiply-add gives exactly; with
//                                  y = RN(1/b), Markstein's theorem gives
//                                  q2 = RN(a/b)
//
// The theorem assumes no step underflows or overflows.  With 2^-50 <= |a|,
// |b| < 2^50 every quotient lies in (2^-100, 2^100) and every remainder near
// 2^(e_a - 24), all normal numbers; dividends or divisors outside that range
// (zeros, subnormals, infinities, NaN) take the IEEE division instead, so
// the result is the bits of a / b (__fdiv_rn) for every input.
// tests/cpp/kdiv_check.cu checks the sequence against the host's IEEE
// division for every fp32 dividend and a set of divisors.
#pragma once

#include <cmath>

namespace tadma_b200 {

struct KnownDivisor {
    float b, y;
    bool ok;  // b inside the range where the fused sequence is exact
};

__host__ __device__ __forceinline__ bool kdiv_in_range(float v) {
    const float m = fabsf(v);
    return m >= 0x1p-50f && m < 0x1p50f;  // false for zeros, subnormals, infinities and NaN
}

#ifdef __CUDA_ARCH__
__device__ __forceinline__ KnownDivisor known_divisor(float b) {
    KnownDivisor d;
    d.b = b;
    d.y = __frcp_rn(b);
    d.ok = kdiv_in_range(b);
    return d;
}
// a / b for a dividend inside the range (kdiv_in_range(a)) and d.ok.
__device__ __forceinline__ float kdiv_fast(float a, const KnownDivisor& d) {
    const float q0 = __fmul_rn(a, d.y);
    const float r0 = __fmaf_rn(-d.b, q0, a);
    const float q1 = __fmaf_rn(r0, d.y, q0);
    const float r1 = __fmaf_rn(-d.b, q1, a);
    return __fmaf_rn(r1, d.y, q1);
}
#else
// Host twin for the exhaustive check: the same steps (fmaf is one rounding;
// built with -ffp-contract=off, so the product stays a rounded multiply).
inline KnownDivisor known_divisor(float b) {
    KnownDivisor d;
    d.b = b;
    d.y = 1.0f / b;
    d.ok = kdiv_in_range(b);
    return d;
}
inline float kdiv_fast(float a, const KnownDivisor& d) {
    const float q0 = a * d.y;
    const float r0 = std::fmaf(-d.b, q0, a);
    const float q1 = std::fmaf(r0, d.y, q0);
    const float r1 = std::fmaf(-d.b, q1, a);
    return std::fmaf(r1, d.y, q1);
}
#endif

}  // namespace tadma_b200
