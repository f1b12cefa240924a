// weights.cu - the weight-file constructor Tensor(std::ifstream&, offset) on
// a file in the generator's layout (raw tensors back to back at cumulative,
// unaligned offsets, cppgen.py:111-116).  Loads every member as a CUDA tensor
// (through the pinned staging ring; the largest spans four slots) and as a
// host tensor, and writes both back to <dir>/<name>.cuda / .cpu.
#include <cstdio>
#include <string>
#include <vector>

#include "tadma/Tadma.hpp"

using namespace tadma;

static std::string g_dir;

template <AnyTensor T>
void dump(const char* name, const char* ext, const T& t) {
    std::vector<char> h((size_t)T::SizeBytes);
    if constexpr (T::device == kCUDA) {
        check_cuda(cudaMemcpyAsync(h.data(), t.data.view, T::SizeBytes, cudaMemcpyDeviceToHost, stream));
        check_cuda(cudaStreamSynchronize(stream));
    } else {
        std::memcpy(h.data(), t.data.view, T::SizeBytes);
    }
    FILE* f = std::fopen((g_dir + "/" + name + "." + ext).c_str(), "wb");
    std::fwrite(h.data(), 1, h.size(), f);
    std::fclose(f);
}

// Members in file order; offsets are the running byte sums.
template <Memory M>
struct Model {
    using A = Allocator<M>;
    std::ifstream bin;
    Tensor<__half, A, Sequence<3, 5, 7>> a;
    Tensor<float, A, Sequence<8192, 1536>> b;  // 48 MiB: four 16 MiB slots, wrapping the ring
    Tensor<int64_t, A, Sequence<129>> c;
    Tensor<__nv_bfloat16, A, Sequence<1000, 3>> d;
    Tensor<double, A, Sequence<17>> e;
    Tensor<float, A, Sequence<4096, 1024>> f;  // 16 MiB: exactly one slot
    explicit Model(const std::string& path)
        : bin(path, std::ios::binary),
          a(bin, 0ULL),
          b(bin, 210ULL),
          c(bin, 50331858ULL),
          d(bin, 50332890ULL),
          e(bin, 50338890ULL),
          f(bin, 50339026ULL) {}
};

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: weights <file.bin> <dir> [cuda]\n");
        return 2;
    }
    g_dir = argv[2];
    {
        Model<kCPU> m(argv[1]);
        dump("a", "cpu", m.a), dump("b", "cpu", m.b), dump("c", "cpu", m.c), dump("d", "cpu", m.d), dump("e", "cpu", m.e),
            dump("f", "cpu", m.f);
    }
    if (argc > 3 && std::string(argv[3]) == "cuda") {
        InitGuard guard;
        Model<kCUDA> m(argv[1]);
        dump("a", "cuda", m.a), dump("b", "cuda", m.b), dump("c", "cuda", m.c), dump("d", "cuda", m.d),
            dump("e", "cuda", m.e), dump("f", "cuda", m.f);
    }
    std::printf("weights ok\n");
    return 0;
}
