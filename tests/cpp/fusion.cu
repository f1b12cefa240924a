// fusion.cu - unchanged generated-code statements (the ONNX LayerNorm
// decomposition and the erf GELU of scripts/generated.cu, with the
// generator's spellings: ConstexprHolder constants, pow<false>, sqrt<true>,
// erf<true>, .template mean<-1>()) run with deferred evaluation on and off.
//
//   fusion check <dir>          writes <dir>/{ln,gelu}_{deferred,eager}.bin
//                               and the inputs; prints "launches <case> <mode> <n>"
//   fusion time <rows> <iters>  prints one JSON line per case and mode
//
// Inputs come from the library's seeded generator (tadma_b200_fill), so the
// oracle regenerates them.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "tadma/Tadma.hpp"

using namespace tadma;

static std::string g_dir;

// Constants the generator emits as static members (cppgen.py:100).
struct Consts {
    static constexpr ConstexprHolder<2.0f> pow_exp = {};
    static constexpr ConstexprHolder<1e-12f> ln_eps = {};
    static constexpr ConstexprHolder<1.4142135381698608f> sqrt2 = {};
    static constexpr ConstexprHolder<1.0f> one = {};
    static constexpr ConstexprHolder<0.5f> half = {};
};

template <AnyTensor T>
void fill(const T& t, int dist, double p0, double p1, uint64_t sid) {
    tadma_tensor d = t.describe_raw();
    detail::check(tadma_b200_fill(&d, dist, p0, p1, 0, sid, 0, stream), "fill");
}

template <AnyTensor T>
void save(const char* name, const T& t) {
    auto h = t.contiguous().template to<kCPU>();
    FILE* f = std::fopen((g_dir + "/" + name + ".bin").c_str(), "wb");
    std::fwrite(h.data.view, sizeof(typename T::ValueType), T::Size, f);
    std::fclose(f);
}

// _bert_embeddings_LayerNorm_* of scripts/generated.cu:652-660 (over the
// last axis, as the ONNX graph means it).
template <AnyTensor X, AnyTensor G, AnyTensor B>
auto layer_norm_block(const X& x, const G& weight, const B& bias) {
    auto ReduceMean_output_0 = x.template mean<-1>();
    auto Sub_output_0 = x - ReduceMean_output_0;
    auto Pow_output_0 = pow<false>(Sub_output_0, Consts::pow_exp);
    auto ReduceMean_1_output_0 = Pow_output_0.template mean<-1>();
    auto Add_output_0 = ReduceMean_1_output_0 + Consts::ln_eps;
    auto Sqrt_output_0 = sqrt<true>(Add_output_0);
    auto Div_output_0 = Sub_output_0 / Sqrt_output_0;
    auto Mul_output_0 = Div_output_0 * weight;
    auto Add_1_output_0 = Mul_output_0 + bias;
    return Add_1_output_0;
}

// The erf form of GELU in ONNX graphs: x * 0.5 * (1 + erf(x / sqrt 2)).
template <AnyTensor X>
auto gelu_block(const X& x) {
    auto Div_output_0 = x / Consts::sqrt2;
    auto Erf_output_0 = erf<true>(Div_output_0);
    auto Add_output_0 = Erf_output_0 + Consts::one;
    auto Mul_output_0 = x * Add_output_0;
    auto Mul_1_output_0 = Mul_output_0 * Consts::half;
    return Mul_1_output_0;
}

template <int64_t R, int64_t H>
struct Inputs {
    Tensor<float, Allocator<kCUDA>, Sequence<R, H>> x;
    Tensor<float, Allocator<kCUDA>, Sequence<H>> g, b;
    Inputs() {
        fill(x, TADMA_DIST_NORMAL, 0.3, 1.0, 1);
        fill(g, TADMA_DIST_NORMAL, 1.0, 0.02, 2);
        fill(b, TADMA_DIST_NORMAL, 0.0, 0.02, 3);
    }
};

void check_mode(bool deferred_on) {
    set_deferred(deferred_on);
    const char* mode = deferred_on ? "deferred" : "eager";
    Inputs<512, 768> in;
    if (deferred_on) {
        save("x", in.x);
        save("gamma", in.g);
        save("beta", in.b);
    }
    check_cuda(cudaStreamSynchronize(stream));
    int64_t before = detail::calls;
    auto ln = layer_norm_block(in.x, in.g, in.b);
    ln.materialize();
    std::printf("launches ln %s %lld\n", mode, (long long)(detail::calls - before));
    save((std::string("ln_") + mode).c_str(), ln);
    before = detail::calls;
    auto ge = gelu_block(in.x);
    ge.materialize();
    std::printf("launches gelu %s %lld\n", mode, (long long)(detail::calls - before));
    save((std::string("gelu_") + mode).c_str(), ge);
}

template <int64_t R>
void time_mode(bool deferred_on, int iters) {
    set_deferred(deferred_on);
    constexpr int64_t H = 768;
    Inputs<R, H> in;
    Tensor<float, Allocator<kCUDA>, Sequence<R, H>> y;
    cudaEvent_t e0, e1;
    check_cuda(cudaEventCreate(&e0));
    check_cuda(cudaEventCreate(&e1));
    const double io_bytes = 2.0 * R * H * 4 + 2.0 * H * 4;  // x read once, y written once (+ gamma, beta)
    for (int which = 0; which < 2; which++) {
        auto step = [&] {
            if (which == 0) y = layer_norm_block(in.x, in.g, in.b);
            else y = gelu_block(in.x);
            y.materialize();
        };
        for (int w = 0; w < 3; w++) step();
        const int64_t before = detail::calls;
        check_cuda(cudaEventRecord(e0, stream));
        for (int i = 0; i < iters; i++) step();
        check_cuda(cudaEventRecord(e1, stream));
        check_cuda(cudaEventSynchronize(e1));
        float ms = 0;
        check_cuda(cudaEventElapsedTime(&ms, e0, e1));
        const double s = ms / 1e3 / iters;
        std::printf("{\"case\": \"%s\", \"mode\": \"%s\", \"rows\": %lld, \"hidden\": %lld, \"us\": %.2f, "
                    "\"launches\": %.1f, \"GBs_io\": %.1f}\n",
                    which == 0 ? "layer_norm block" : "erf gelu block", deferred_on ? "deferred" : "eager",
                    (long long)R, (long long)H, s * 1e6, (double)(detail::calls - before) / iters,
                    (which == 0 ? io_bytes : 2.0 * R * H * 4) / s / 1e9);
    }
}

int main(int argc, char** argv) {
    if (argc < 3) {
        std::fprintf(stderr, "usage: fusion check <dir> | fusion time <rows> <iters>\n");
        return 2;
    }
    InitGuard guard;
    if (std::strcmp(argv[1], "check") == 0) {
        g_dir = argv[2];
        check_mode(true);
        check_mode(false);
    } else {
        const int iters = argc > 3 ? std::atoi(argv[3]) : 20;
        // 65536 rows x 768: x and y are 201 MB each, larger than L2
        time_mode<65536>(true, iters);
        time_mode<65536>(false, iters);
    }
    check_cuda(cudaStreamSynchronize(stream));
    std::printf("fusion ok\n");
    return 0;
}
