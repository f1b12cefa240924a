// Host-side fault injection in the header API's device allocator: with
// TADMA_B200_FAIL_ALLOC=1 constructing a CUDA tensor throws std::runtime_error
// (the reference's check_cuda convention, Defines.hpp:14-26) before any CUDA
// call is made, so this program needs no GPU.
#include <cstdio>
#include <cstdlib>

#include "tadma/Tadma.hpp"

using namespace tadma;

int main() {
    setenv("TADMA_B200_FAIL_ALLOC", "1", 1);
    try {
        Tensor<float, Allocator<kCUDA>, Sequence<4, 8>> t;
        std::printf("no exception\n");
        return 1;
    } catch (const std::runtime_error& e) {
        std::printf("caught: %s\n", e.what());
    }
    // A tensor without elements allocates nothing and is still created.
    Tensor<float, Allocator<kCUDA>, Sequence<0, 8>> empty;
    std::printf("empty tensor ok: %p\n", static_cast<void*>(empty.data.view));
    return 0;
}
