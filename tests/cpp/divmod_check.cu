// Host-side check of the index divider in tadma_b200/csrc/common.cuh
// (DivMod): the 64-bit and the 32-bit magic-multiplier quotients against
// exact division, for every small divisor, the powers of two and their
// neighbours, and pseudo-random divisors, each with edge and pseudo-random
// dividends.  The device paths run the same formulas (__umul64hi / __umulhi
// in place of the host's wide multiplies).  Prints "ok" and exits 0 on success.
#include <cstdio>
#include <vector>

#include "../../tadma_b200/csrc/common.cuh"

static uint64_t next(uint64_t& s) {  // splitmix64
    uint64_t z = (s += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

int main() {
    std::vector<uint64_t> ds;
    for (uint64_t d = 1; d <= 4096; d++) ds.push_back(d);
    for (int k = 1; k < 64; k++)
        for (int o = -1; o <= 1; o++) ds.push_back((1ull << k) + o);
    uint64_t s = 7;
    for (int i = 0; i < 4000; i++) ds.push_back(next(s) >> (next(s) % 64) | 1);
    long checks = 0;
    for (uint64_t d : ds) {
        if (d == 0) continue;
        tadma_b200::DivMod dm(d);
        std::vector<uint64_t> ns = {0, 1, d - 1, d, d + 1, ~0ull, ~0ull - 1, 0xffffffffull, 0xfffffffeull};
        for (int i = 0; i < 64; i++) ns.push_back(next(s) >> (next(s) % 64));
        for (uint64_t n : ns) {
            uint64_t q, r;
            dm.divmod(n, q, r);
            if (q != n / d || r != n % d) {
                std::printf("64-bit: %llu / %llu\n", (unsigned long long)n, (unsigned long long)d);
                return 1;
            }
            if (d <= 0xffffffffull && n <= 0xffffffffull) {
                const uint32_t q32 = dm.div32((uint32_t)n);
                if (q32 != n / d) {
                    std::printf("32-bit: %llu / %llu\n", (unsigned long long)n, (unsigned long long)d);
                    return 1;
                }
            }
            checks++;
        }
    }
    std::printf("ok %ld\n", checks);
    return 0;
}
