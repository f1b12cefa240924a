// tape.cu - the ExecutionTape / node layer of the header API (Node.hpp,
// ExecutionTape.hpp, NodeOps.hpp), run on CUDA tensors ("cuda") or host
// tensors ("cpu", no GPU needed).  Every result is written to <dir>/<name>.bin
// (row-major float32) and checked by tests/test_tape*.py; the merged node
// counts are printed as "nodes <case> <n>".
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "tadma/Tadma.hpp"

using namespace tadma;

static std::string g_dir;

template <AnyTensor T>
void write(const char* name, const T& t) {
    using V = typename T::ValueType;
    std::vector<V> h((size_t)T::Size);
    if constexpr (T::device == kCUDA) {
        auto c = t.contiguous();
        check_cuda(cudaMemcpyAsync(h.data(), c.data.view, sizeof(V) * T::Size, cudaMemcpyDeviceToHost, stream));
        check_cuda(cudaStreamSynchronize(stream));
    } else {
        for (int64_t i = 0; i < T::Size; i++) h[i] = t[i];
    }
    std::string path = g_dir + "/" + name + ".bin";
    FILE* f = std::fopen(path.c_str(), "wb");
    std::fwrite(h.data(), sizeof(V), h.size(), f);
    std::fclose(f);
}

// A functor struct with a declared device capability.
struct CosIndex {
    static constexpr bool tadma_device = true;
    __host__ __device__ float operator()(int64_t i) const { return cosf(0.37f * (float)i); }
};

// A plain aggregate functor: device-capable as is.
struct Fma {
    float a;
    __host__ __device__ void operator()(const float& x, const float& y, float& z) const { z = a * x + y; }
};

struct RampIndex {
    static constexpr bool tadma_device = true;
    __host__ __device__ float operator()(int64_t i) const { return (float)(i % 13) - 6.0f; }
};

template <typename Tape>
void count(const char* name, const Tape&) {
    std::printf("nodes %s %d\n", name, (int)Tape::Size);
}

template <Memory M>
void run() {
    auto noop = [](const auto&...) {};

    // 1. A chain of operators on tape tensors: one merged node (the index
    //    node's functor is device-capable and every shared tensor is elementwise).
    {
        ExecutionTape tape;
        auto [t1, a] = tape.Append(index_to_value<Sequence<64, 96>, M>(CosIndex{}));
        auto [t2, b] = t1.Append(a * 3.0f);
        auto [t3, c] = t2.Append(b + 1.5f);
        auto [t4, d] = t3.Append(c * a);
        auto [t5, e] = t4.Append(sigmoid(d));  // in place: e aliases d
        auto [t6, f] = t5.Append(e - b);
        auto [t7] = t6.Append(make_node<Sequence<>>(noop, f, a));
        auto g = t7.Optimize();
        count("chain", g);
        g.Evaluate(0);
        write("chain_a", std::get<1>(g.Last().tensors));
        write("chain_f", std::get<0>(g.Last().tensors));
    }
    // 2. An unannotated lambda: nvcc compiles it for the host only, so its
    //    node runs on the host; the operator node after it runs on the device.
    {
        ExecutionTape tape;
        auto [t1, a] = tape.Append(index_to_value<Sequence<50, 40>, M>([](float i) -> float { return i * 0.5f - 7.0f; }));
        auto [t2, b] = t1.Append(a * 2.0f);
        auto [t3, c] = t2.Append(-b);
        auto [t4, o] = t3.Append(make_node<Sequence<>>(noop, c));
        auto g = t4.Optimize();
        count("host_lambda", g);
        g.Evaluate(0);
        write("host_lambda_c", std::get<0>(g.Last().tensors));
    }
    // 3. A transposed read of a tape tensor is not merged into its producer
    //    (another thread writes the element it reads).
    {
        ExecutionTape tape;
        auto [t1, p] = tape.Append(index_to_value<Sequence<48, 80>, M>(RampIndex{}));
        auto pt = p.template transpose<1, 0>();
        auto [t2, q] = t1.Append(pt * 2.0f);
        auto [t3] = t2.Append(make_node<Sequence<>>(noop, q, p));
        auto g = t3.Optimize();
        count("transposed", g);
        g.Evaluate(0);
        write("transposed_p", std::get<1>(g.Last().tensors));
        write("transposed_q", std::get<0>(g.Last().tensors));
    }
    // 4. CombineVariadicNode with a user functor, y broadcast over x's rows.
    {
        Tensor<float, Allocator<M>, Sequence<32, 256>> x, z;
        Tensor<float, Allocator<M>, Sequence<256>> y;
        make_node<Sequence<32 * 256>>(nodefn::IndexToValue<CosIndex>(CosIndex{}), x).Evaluate(0);
        make_node<Sequence<256>>(nodefn::IndexToValue<RampIndex>(RampIndex{}), y).Evaluate(0);
        auto node = CombineVariadicNode(Fma{2.5f}, x, y, z);
        node.Evaluate(0);
        write("fma_x", x);
        write("fma_y", y);
        write("fma_z", z);
#ifdef __CUDACC_EXTENDED_LAMBDA__
        // 5. An extended lambda (nvcc --extended-lambda) runs on the device.
        Tensor<float, Allocator<M>, Sequence<32, 256>> w;
        auto sq = CombineVariadicNode([] __host__ __device__(const float& v, float& r) { r = v * v - 1.0f; }, x, w);
        sq.Evaluate(0);
        write("lambda_w", w);
        std::printf("extended lambda ok\n");
#endif
    }
}

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: tape cuda|cpu <dir>\n");
        return 2;
    }
    g_dir = argv[2];
    if (std::strcmp(argv[1], "cuda") == 0) {
        InitGuard guard;
        run<kCUDA>();
        check_cuda(cudaStreamSynchronize(stream));
    } else {
        run<kCPU>();
    }
    std::printf("tape ok\n");
    return 0;
}
