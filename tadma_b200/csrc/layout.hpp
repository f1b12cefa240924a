// layout.hpp - run-time shape/stride folding shared by every engine.
//
// The reference folds layouts at compile time: removeFakeDims drops size-1 /
// stride-0 dims and removeContiguousDims merges dims that are contiguous with
// their inner neighbour (Tensor.hpp:242-273); its executors then ignore the
// result and pay a div/mod per dim per element (Node.hpp:25-35 via
// Utils.hpp:9-17).  Here the folded layout drives kernel selection: after
// folding, most element-wise launches are rank 1 (pure streaming) or rank 2
// (a row broadcast such as bias[cols] over x[rows, cols]).
#pragma once

#include <stdint.h>

#include "../../include/tadma_b200.h"

namespace tadma_b200 {

// Joint layout of up to 1 + TADMA_MAX_INPUTS operands over one shape.
struct Folded {
    int rank = 0;                                   // >= 1 after fold()
    int64_t dims[TADMA_MAX_RANK] = {};              // row-major, outermost first
    int64_t strides[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK] = {};  // [0] = out
};

// Fold `nops` operands that all have logical shape dims[0..rank).  Operand k's
// strides are strides[k]; a dim where operand k has extent 1 must already have
// stride 0 there.  Dims of extent 1 are dropped; adjacent dims d, d+1 merge
// when every operand has stride[d] == stride[d+1] * dims[d+1].
inline Folded fold(int rank, const int64_t* dims, const int64_t (*strides)[TADMA_MAX_RANK], int nops) {
    Folded f;
    // Drop extent-1 dims.
    int64_t D[TADMA_MAX_RANK];
    int64_t S[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    int r = 0;
    for (int d = 0; d < rank; d++) {
        if (dims[d] == 1) continue;
        D[r] = dims[d];
        for (int k = 0; k < nops; k++) S[k][r] = strides[k][d];
        r++;
    }
    if (r == 0) {
        f.rank = 1;
        f.dims[0] = 1;
        for (int k = 0; k < nops; k++) f.strides[k][0] = 1;
        return f;
    }
    // Merge from the innermost dim outwards.
    int out_r = 0;
    int64_t FD[TADMA_MAX_RANK];
    int64_t FS[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    // Build in reverse (innermost first), then flip.
    FD[0] = D[r - 1];
    for (int k = 0; k < nops; k++) FS[k][0] = S[k][r - 1];
    out_r = 1;
    for (int d = r - 2; d >= 0; d--) {
        bool mergeable = true;
        for (int k = 0; k < nops; k++)
            if (S[k][d] != FS[k][out_r - 1] * FD[out_r - 1]) mergeable = false;
        if (mergeable) {
            FD[out_r - 1] *= D[d];
        } else {
            FD[out_r] = D[d];
            for (int k = 0; k < nops; k++) FS[k][out_r] = S[k][d];
            out_r++;
        }
    }
    f.rank = out_r;
    for (int i = 0; i < out_r; i++) {
        f.dims[i] = FD[out_r - 1 - i];
        for (int k = 0; k < nops; k++) f.strides[k][i] = FS[k][out_r - 1 - i];
    }
    return f;
}

}  // namespace tadma_b200
