// Host-side check of the shared-divisor division in
// tadma_b200/csrc/kdiv.cuh: for each divisor b of a set (simple values, the
// significands next to 1 and 2, the range ends, pseudo-random ones, both
// signs), every fp32 dividend a inside the fast range is divided by the
// reciprocal sequence and compared, bit for bit, with the host's IEEE
// division a / b; then pseudo-random (a, b) pairs across the whole range.
// The device runs the same steps (__fmul_rn, __fmaf_rn, __frcp_rn).  Prints
// "ok" and exits 0 when no quotient differs.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../tadma_b200/csrc/kdiv.cuh"

using tadma_b200::KnownDivisor;

static float bits_f(uint32_t u) {
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
static uint32_t f_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
static uint64_t next(uint64_t& s) {  // splitmix64
    uint64_t z = (s += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Mismatches over every dividend of the fast range for one divisor.
static long all_dividends(float b) {
    const KnownDivisor d = tadma_b200::known_divisor(b);
    if (!d.ok) return 0;
    long bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static)
    for (int64_t hi = 0; hi < 65536; hi++) {
        for (uint32_t lo = 0; lo < 65536; lo++) {
            const float a = bits_f((uint32_t)(hi << 16) | lo);
            const bool in = tadma_b200::kdiv_in_range(a);
            const uint32_t got = f_bits(tadma_b200::kdiv_fast(a, d));
            const uint32_t want = f_bits(a / b);
            bad += (in && got != want) ? 1 : 0;
        }
    }
    return bad;
}

int main() {
    std::vector<float> bs = {1.0f, 2.0f, 3.0f, 5.0f, 7.0f, 10.0f, 0.1f, 1.0f / 3.0f, 1.41421354f, 0.70710677f,
                             bits_f(0x3f800001u), bits_f(0x3fffffffu), bits_f(0x3ffffffeu), bits_f(0x3fc00001u),
                             0x1p-50f, bits_f(0x587fffffu) /* largest below 2^50 */, 1e-12f, 6.02e14f};
    uint64_t s = 11;
    for (int i = 0; i < 12; i++) {
        // a pseudo-random significand with an exponent in [-50, 49]
        const uint32_t e = 127 - 50 + (uint32_t)(next(s) % 100);
        bs.push_back(bits_f((e << 23) | (uint32_t)(next(s) & 0x7fffff)));
    }
    const size_t n0 = bs.size();
    for (size_t i = 0; i < n0; i += 3) bs.push_back(-bs[i]);
    long checked = 0;
    for (float b : bs) {
        const long bad = all_dividends(b);
        if (bad) {
            std::printf("divisor %a: %ld quotients differ\n", b, bad);
            return 1;
        }
        checked++;
    }
    // pseudo-random pairs inside the range
    long bad = 0, pairs = 0;
#pragma omp parallel for reduction(+ : bad, pairs) schedule(static)
    for (int t = 0; t < 64; t++) {
        uint64_t r = 1000 + t;
        for (int i = 0; i < (1 << 22); i++) {
            const uint64_t z = next(r);
            const uint32_t ea = 127 - 50 + (uint32_t)(z % 100), eb = 127 - 50 + (uint32_t)((z >> 8) % 100);
            const uint64_t w = next(r);
            const float a = bits_f((uint32_t)(z >> 63) << 31 | ea << 23 | (uint32_t)(w & 0x7fffff));
            const float b = bits_f((uint32_t)((z >> 62) & 1) << 31 | eb << 23 | (uint32_t)((w >> 23) & 0x7fffff));
            const KnownDivisor d = tadma_b200::known_divisor(b);
            bad += f_bits(tadma_b200::kdiv_fast(a, d)) != f_bits(a / b);
            pairs++;
        }
    }
    if (bad) {
        std::printf("%ld of %ld random pairs differ\n", bad, pairs);
        return 1;
    }
    std::printf("ok: %ld divisors x all dividends, %ld random pairs\n", checked, pairs);
    return 0;
}
