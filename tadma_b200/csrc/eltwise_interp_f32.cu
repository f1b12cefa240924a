// eltwise_interp_f32.cu - the interpreted chain kernels in fp32 compute
// (precise and fast math), instantiated for 0..6 operands.
#include "eltwise_impl.cuh"

namespace tadma_b200 {
namespace {



}  // namespace

int launch_interp_f32(int nin, bool fast, const ChainParams& p, bool vec, int64_t work, cudaStream_t s, bool narrow) {
    if (fast) {
        switch (nin) {
        case 0: return launch<float, 0, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        case 1: return launch<float, 1, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        case 2: return launch<float, 2, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        case 3: return launch<float, 3, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        case 4: return launch<float, 4, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        case 5: return launch<float, 5, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        default: return launch<float, 6, PROG_INTERP_FAST>(p, vec, work, s, narrow);
        }
    }
    switch (nin) {
    case 0: return launch<float, 0, PROG_INTERP>(p, vec, work, s, narrow);
    case 1: return launch<float, 1, PROG_INTERP>(p, vec, work, s, narrow);
    case 2: return launch<float, 2, PROG_INTERP>(p, vec, work, s, narrow);
    case 3: return launch<float, 3, PROG_INTERP>(p, vec, work, s, narrow);
    case 4: return launch<float, 4, PROG_INTERP>(p, vec, work, s, narrow);
    case 5: return launch<float, 5, PROG_INTERP>(p, vec, work, s, narrow);
    default: return launch<float, 6, PROG_INTERP>(p, vec, work, s, narrow);
    }
}

}  // namespace tadma_b200
