// eltwise_interp_wide.cu - the interpreted chain kernels in fp64 and int64
// compute, instantiated for 0..6 operands.
#include "eltwise_impl.cuh"

namespace tadma_b200 {
namespace {

template <typename C>
int launch_wide(int nin, const ChainParams& p, bool vec, int64_t work, cudaStream_t s) {
    switch (nin) {
    case 0: return launch<C, 0, PROG_INTERP>(p, vec, work, s);
    case 1: return launch<C, 1, PROG_INTERP>(p, vec, work, s);
    case 2: return launch<C, 2, PROG_INTERP>(p, vec, work, s);
    case 3: return launch<C, 3, PROG_INTERP>(p, vec, work, s);
    case 4: return launch<C, 4, PROG_INTERP>(p, vec, work, s);
    case 5: return launch<C, 5, PROG_INTERP>(p, vec, work, s);
    default: return launch<C, 6, PROG_INTERP>(p, vec, work, s);
    }
}

}  // namespace

int launch_interp_f64(int nin, const ChainParams& p, bool vec, int64_t work, cudaStream_t s) {
    return launch_wide<double>(nin, p, vec, work, s);
}

int launch_interp_i64(int nin, const ChainParams& p, bool vec, int64_t work, cudaStream_t s) {
    return launch_wide<int64_t>(nin, p, vec, work, s);
}

}  // namespace tadma_b200
