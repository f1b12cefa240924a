// eltwise_affine.cu - compile-time affine + activation programs act(x * s [+ y])
// on the chain kernels (fp32 compute).
#include "eltwise_impl.cuh"

namespace tadma_b200 {
namespace {

// Affine + activation vector kernels (fp32 compute).
template <int ACT, bool FAST, bool MUL>
int launch_affine_add(bool add, const ChainParams& p, int64_t work, cudaStream_t s, bool narrow) {
    if (add) return launch<float, 2, affine_prog(ACT, FAST, MUL, true)>(p, true, work, s, narrow);
    return launch<float, 1, affine_prog(ACT, FAST, MUL, false)>(p, true, work, s, narrow);
}
template <int ACT, bool FAST>
int launch_affine_mul(bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s, bool narrow) {
    return mul ? launch_affine_add<ACT, FAST, true>(add, p, work, s, narrow)
               : launch_affine_add<ACT, FAST, false>(add, p, work, s, narrow);
}
template <int ACT>
int launch_affine_fast(bool fast, bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s, bool narrow) {
    return fast ? launch_affine_mul<ACT, true>(mul, add, p, work, s, narrow)
                : launch_affine_mul<ACT, false>(mul, add, p, work, s, narrow);
}

}  // namespace

int launch_affine(int act, bool fast, bool mul, bool add, const ChainParams& p, int64_t work, cudaStream_t s,
                  bool narrow) {
    switch (act) {
    case ACT_GELU: return launch_affine_fast<ACT_GELU>(fast, mul, add, p, work, s, narrow);
    case ACT_RELU: return launch_affine_fast<ACT_RELU>(fast, mul, add, p, work, s, narrow);
    case ACT_SIGMOID: return launch_affine_fast<ACT_SIGMOID>(fast, mul, add, p, work, s, narrow);
    case ACT_TANH: return launch_affine_fast<ACT_TANH>(fast, mul, add, p, work, s, narrow);
    default: return launch_affine_fast<ACT_NONE>(fast, mul, add, p, work, s, narrow);
    }
}

}  // namespace tadma_b200
