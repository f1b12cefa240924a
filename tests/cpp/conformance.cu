// Conformance program for the header-only Tensor API (include/tadma/Tadma.hpp):
// calls written the way TADMA's generated graph code writes them
// (scripts/generated.cu style: operators, .template mean<...>(), pow<false>,
// sqrt<true>, softmax<-1,false>, gather, concat, transpose, slice, unsqueeze,
// reshape, where, to<T>), on seeded synthetic inputs.  Every result is written
// as raw bytes to <outdir>/<name>.bin; tests/test_cpp_api_gpu.py regenerates
// the inputs with the oracle and checks each file.
//
// Build: nvcc -std=c++20 -gencode arch=compute_100a,code=sm_100a -I include
//        tests/cpp/conformance.cu -L tadma_b200 -ltadma_b200
#include <cstdio>
#include <string>

#include "tadma/Tadma.hpp"

using namespace tadma;
using ALLOCATOR = Allocator<kCUDA>;

static std::string g_dir;

// The embedding prologue of a generated BERT-style graph, written the way the
// generator writes it: constants are types (ConstexprHolder, a
// ConstexprAllocator position table), the Shape / Gather / Unsqueeze / Concat
// / Mul / Equal / Where arithmetic on shapes folds at compile time, and only
// the tensor work launches kernels.
struct GraphPrologue {
    static constexpr ConstexprHolder<1> c_one = {};
    static constexpr ConstexprHolder<0> c_zero = {};
    static constexpr ConstexprHolder<-1> c_minus1 = {};
    static constexpr ConstexprHolder<2.0> c_two = {};
    using position_seq = Sequence<0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15>;
    Tensor<TYPE(position_seq::Array()[0]), ConstexprAllocator<position_seq>, Sequence<16>> position_ids = {};
    Tensor<float, Allocator<kCUDA>, Sequence<16, 32>> position_table;

    template <int64_t B, int64_t S>
    auto infer(const Tensor<int64_t, Allocator<kCUDA>, Sequence<B, S>>& input_ids,
               const Tensor<float, Allocator<kCUDA>, Sequence<100, 32>>& word_table) {
        auto shp = shape(input_ids);                      // [B, S]
        auto seq = gather(shp, c_one);                    // S
        auto seq1 = seq.template unsqueeze<c_zero>();     // [S]
        constexpr int64_t seq_len = seq1;
        static_assert(seq_len == S);
        auto pid = position_ids.template slice<c_zero, seq1, 0, c_one>();  // the first S positions
        auto word = gather(word_table, input_ids);        // [B, S, 32]
        auto pos = gather(position_table, pid);           // [S, 32]
        auto emb = word + pos;                            // [B, S, 32]
        auto new_shape = concat<0>(gather(shp, c_zero), c_minus1);  // [B, -1]
        auto flat = emb.template reshape<new_shape>();    // [B, S * 32]
        static_assert(decltype(flat)::Dim(0) == B && decltype(flat)::Dim(1) == S * 32);
        auto dims = shp * c_one;                          // [B, S]
        auto is_unknown = dims == c_minus1;               // [false, false]
        auto fixed = where(is_unknown, c_one, dims);      // [B, S]
        static_assert(decltype(fixed)::at(0) == B && decltype(fixed)::at(1) == S);
        static_assert(decltype(c_two * c_two)::value == 4.0);
        auto expanded = pos.template broadcastTo<TYPE(emb)>().contiguous();  // Expand to [B, S, 32]
        return std::make_tuple(pid.contiguous(), flat, expanded);
    }
};

template <AnyTensor T>
void fill(const T& t, int dist, double p0, double p1, uint64_t sid) {
    tadma_tensor d = t.describe();
    detail::check(tadma_b200_fill(&d, dist, p0, p1, 0, sid, 0, stream), "fill");
}

template <AnyTensor T>
void save(const char* name, const T& t) {
    auto h = t.contiguous().template to<kCPU>();
    std::string path = g_dir + "/" + name + ".bin";
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) throw std::runtime_error("cannot write " + path);
    std::fwrite(h.data.view, sizeof(typename T::ValueType), T::Size, f);
    std::fclose(f);
}

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s <outdir>\n", argv[0]);
        return 2;
    }
    g_dir = argv[1];
    InitGuard guard;

    // config 2 through the operators: x * 0.5f -> float, + bias -> float, gelu in place.
    Tensor<__nv_bfloat16, ALLOCATOR, Sequence<64, 1024>> x;
    Tensor<__nv_bfloat16, ALLOCATOR, Sequence<1024>> bias;
    fill(x, TADMA_DIST_NORMAL, 0.0, 1.0, 1);
    fill(bias, TADMA_DIST_NORMAL, 0.0, 0.1, 2);
    auto y_ops = gelu(x * 0.5f + bias);
    static_assert(std::is_same_v<decltype(y_ops)::ValueType, float>);
    save("cfg2_ops_f32", y_ops);
    // config 2 as one fused kernel with a bf16 result.
    auto y_fused = fused<__nv_bfloat16>(x, fuse::mul(0.5), fuse::add(bias), fuse::gelu());
    save("cfg2_fused_bf16", y_fused);

    // config 1: y = sum_{last}(exp(A + b)), A[64,128], b[128] fp32.
    Tensor<float, ALLOCATOR, Sequence<64, 128>> A;
    Tensor<float, ALLOCATOR, Sequence<128>> b;
    fill(A, TADMA_DIST_NORMAL, 0.0, 1.0, 1);
    fill(b, TADMA_DIST_NORMAL, 0.0, 1.0, 2);
    auto e = exp<false>(A + b);
    auto s1 = e.template sum<-1, false>();
    static_assert(decltype(s1)::Rank == 1 && decltype(s1)::Dim(0) == 64);
    save("cfg1_sum", s1);
    // config 1 as one kernel: the chain add-then-exp reduced where it is computed
    auto s1f = fused_reduce<TADMA_REDUCE_SUM, -1, false>(A, fuse::add(b), fuse::exp());
    static_assert(std::is_same_v<decltype(s1f)::ValueType, float> && decltype(s1f)::Dim(0) == 64);
    save("cfg1_fused_sum", s1f);

    // config 3 (scaled): X[2, 64, 256] ~ U(-1, 1).
    Tensor<float, ALLOCATOR, Sequence<2, 64, 256>> X;
    fill(X, TADMA_DIST_UNIFORM, -1.0, 1.0, 3);
    save("cfg3_sum", X.template sum<-1>());
    save("cfg3_max", X.template max<-1>());
    save("cfg3_argmax", X.template argmax<-1>());
    save("cfg3_mean1", X.template mean<1>());

    // config 4 (scaled): ONNX LayerNorm and softmax, fp16.
    Tensor<__half, ALLOCATOR, Sequence<4, 16, 1024>> L;
    Tensor<__half, ALLOCATOR, Sequence<1024>> g, be;
    fill(L, TADMA_DIST_NORMAL, 0.0, 1.0, 4);
    fill(g, TADMA_DIST_NORMAL, 1.0, 0.02, 5);
    fill(be, TADMA_DIST_NORMAL, 0.0, 0.02, 6);
    save("cfg4_ln", layer_norm_onnx<-1, false>(L, g, be, 1e-5f));
    save("cfg4_ln_tadma", layer_norm<-1, false>(L, g, be, 1e-5f));
    Tensor<__half, ALLOCATOR, Sequence<2, 4, 256, 2048>> S;
    fill(S, TADMA_DIST_NORMAL, 0.0, 3.0, 7);
    save("cfg4_softmax", softmax<-1, false>(S));

    // config 5 (scaled): embedding gather + position table, fused and as two ops.
    Tensor<__half, ALLOCATOR, Sequence<1000, 256>> table;
    Tensor<int64_t, ALLOCATOR, Sequence<4, 64>> ids;
    Tensor<__nv_bfloat16, ALLOCATOR, Sequence<64, 256>> pos;
    fill(table, TADMA_DIST_NORMAL, 0.0, 0.02, 8);
    fill(ids, TADMA_DIST_INDEX, 0.0, 1000.0, 9);
    fill(pos, TADMA_DIST_NORMAL, 0.0, 0.02, 10);
    auto emb = gather_add(table, ids, pos);
    static_assert(std::is_same_v<decltype(emb)::ValueType, float>);
    save("cfg5_gather_add_f32", emb);
    auto gathered = gather(table, ids);
    save("cfg5_gather", gathered);

    // generated.cu's decomposed LayerNorm chain (ReduceMean, Sub, Pow 2,
    // ReduceMean, Add eps, Sqrt, Div, Mul, Add) on [2, 8, 768] fp32.
    Tensor<float, ALLOCATOR, Sequence<2, 8, 768>> h;
    Tensor<float, ALLOCATOR, Sequence<768>> w, wb;
    fill(h, TADMA_DIST_NORMAL, 0.0, 1.0, 11);
    fill(w, TADMA_DIST_NORMAL, 1.0, 0.02, 12);
    fill(wb, TADMA_DIST_NORMAL, 0.0, 0.02, 13);
    auto m = h.template mean<-1>();
    auto sub = h - m;
    auto sq = pow<false>(sub, 2.0f);
    auto var = sq.template mean<-1>();
    auto ve = var + 9.999999960041972e-13;
    auto sd = sqrt<true>(ve);
    auto nrm = sub / sd;
    auto mul = nrm * w;
    auto ln = mul + wb;
    save("gen_ln", ln);

    // views and copies
    auto tr = X.template transpose<0, 2, 1>().contiguous();
    static_assert(decltype(tr)::Dim(1) == 256 && decltype(tr)::Dim(2) == 64);
    save("view_transpose", tr);
    auto sl = X.template slice<1, 9, 1, 2>().contiguous();  // rows 1, 3, 5, 7 of axis 1
    static_assert(decltype(sl)::Dim(1) == 4);
    save("view_slice", sl);
    auto rs = X.template reshape<2, -1>();
    static_assert(decltype(rs)::Dim(1) == 64 * 256);
    save("view_reshape_sum", rs.template sum<1, false>());
    auto cc = concat<1>(X, X.template slice<0, 8, 1>());
    static_assert(decltype(cc)::Dim(1) == 72);
    save("concat", cc);
    auto cond = X > 0.25f;
    auto wsel = where(cond, X, X * -1.0f);
    save("where", wsel);
    save("cast_f16", X.template to<__half>());
    auto un = b.template unsqueeze<0>();  // [1, 128]
    save("unsqueeze_bcast_add", A + un);

    // lazy chains (Lazy.hpp): each pair is the same computation made through
    // lazy values (one kernel where consumed) and eagerly (one kernel per op);
    // the test compares them bit for bit.
    Tensor<float, ALLOCATOR, Sequence<64, 128>> A2, A3, A4, A5;
    fill(A2, TADMA_DIST_NORMAL, 0.0, 1.0, 17);
    fill(A3, TADMA_DIST_NORMAL, 0.0, 1.0, 18);
    fill(A4, TADMA_DIST_NORMAL, 0.0, 1.0, 19);
    fill(A5, TADMA_DIST_NORMAL, 0.0, 1.0, 20);
    {
        auto l2 = gelu(lazy(x) * 0.5f + bias);  // config 2: float chain, gelu in place
        static_assert(LazyTensor<decltype(l2)> && std::is_same_v<decltype(l2)::ValueType, float>);
        save("lazy_cfg2", l2);
        save("eager_cfg2", gelu(x * 0.5f + bias));
        auto l2d = gelu<false>(lazy(x) * 0.5f + bias);  // double result: the chain restarts at gelu
        static_assert(std::is_same_v<decltype(l2d)::ValueType, double>);
        save("lazy_cfg2_f64", l2d);
        save("eager_cfg2_f64", gelu<false>(x * 0.5f + bias));

        auto l1 = exp<false>(lazy(A) + b).template sum<-1, false>();  // config 1 in one kernel
        static_assert(std::is_same_v<decltype(l1)::ValueType, float> && decltype(l1)::Rank == 1 && decltype(l1)::Dim(0) == 64);
        save("lazy_cfg1_sum", l1);

        auto lm = lazy(X) * 2.0f - 0.5f;
        save("lazy_max", lm.template max<-1>());
        save("eager_max", (X * 2.0f - 0.5f).template max<-1>());
        save("lazy_argmin1", lm.template argmin<1>());
        save("eager_argmin1", (X * 2.0f - 0.5f).template argmin<1>());

        // every operator with a lazy operand extends a chain (no eager kernel)
        static_assert(LazyTensor<decltype(lm)> && LazyTensor<decltype(-lazy(A))>);
        static_assert(LazyTensor<decltype((A2 - lazy(A)) / (1.0f + lazy(A3)) + A4 / lazy(A))>);
        static_assert(LazyTensor<decltype((A2 > lazy(A)) && (lazy(A3) < 0.5f))>);
        static_assert(LazyTensor<decltype(lazy(A) + A2 - A3 + A4 - A5)>);
        static_assert(LazyTensor<decltype(pow<false>(sqrt(lazy(A)), 2.0f))>);
        static_assert(!LazyTensor<decltype(A + A2)>);
        save("lazy_rev", (A2 - lazy(A)) / (1.0f + lazy(A3)) + A4 / lazy(A));
        save("eager_rev", (A2 - A) / (1.0f + A3) + A4 / A);
        save("lazy_cmp", (A2 > lazy(A)) && (lazy(A3) < 0.5f));
        save("eager_cmp", (A2 > A) && (A3 < 0.5f));

        auto li = lazy(ids) * 3 + 1;  // integer chain
        static_assert(std::is_same_v<decltype(li)::ValueType, int64_t>);
        save("lazy_int", (li > 1500) * 2.5);
        save("eager_int", ((ids * 3 + 1) > 1500) * 2.5);

        auto ll = lazy(A);  // 20 steps: more than one chain's 16 instructions
        auto le = A.clone();
        for (int i = 0; i < 10; i++) {
            ll *= 1.0625f;
            ll += A2;
            le *= 1.0625f;
            le += A2;
        }
        save("lazy_long", ll);
        save("eager_long", le);
        save("lazy_operands", lazy(A) + A2 - A3 + A4 - A5);  // 4 tensor operands: more than 3
        save("eager_operands", A + A2 - A3 + A4 - A5);
        save("lazy_square", lazy(A) * A + A2 * lazy(A2));  // operands that are the source
        save("eager_square", A * A + A2 * A2);

        // where with a lazy condition: one step reading both branches
        auto lw = where(lazy(A) > A2, A3, lazy(A4) * 2.0f);
        static_assert(LazyTensor<decltype(lw)> && std::is_same_v<decltype(lw)::ValueType, float>);
        save("lazy_where", lw + 1.0f);
        save("eager_where", where(A > A2, A3, A4 * 2.0f) + 1.0f);
        save("lazy_where_sum", where(lazy(X) < 0.0f, X * 0.5f, X).template sum<-1>());
        save("eager_where_sum", where(X < 0.0f, X * 0.5f, X).template sum<-1>());
        save("lazy_softmax", softmax<-1, false>(lazy(S) * 0.5f));  // consumed by an eager API call
        save("eager_softmax", softmax<-1, false>(S * 0.5f));
        // an in-place call materialises the lazy value and writes there; later
        // steps and reductions start from that tensor
        auto ls = softmax<-1, true>(lazy(S) * 0.5f);
        save("lazy_softmax_then", (ls * 3.0f).template max<-1>());
        auto es = softmax<-1, true>(S * 0.5f);
        save("eager_softmax_then", (es * 3.0f).template max<-1>());
        save("lazy_cast_sum", tanh(lazy(L).template to<float>()).template sum<-1>());
        save("eager_cast_sum", tanh(L.template to<float>()).template sum<-1>());
    }

    // generated-graph shape arithmetic (GraphPrologue above)
    GraphPrologue graph;
    fill(graph.position_table, TADMA_DIST_NORMAL, 0.0, 1.0, 15);
    Tensor<float, ALLOCATOR, Sequence<100, 32>> word_table;
    // infer() deduces <B, S> as int64_t, so the dims are spelled as int64_t values
    Tensor<int64_t, ALLOCATOR, Sequence<int64_t(2), int64_t(12)>> input_ids;
    fill(word_table, TADMA_DIST_NORMAL, 0.0, 1.0, 14);
    fill(input_ids, TADMA_DIST_INDEX, 0.0, 100.0, 16);
    auto [pid, flat, expanded] = graph.infer(input_ids, word_table);
    save("gen_position_ids", pid);
    save("gen_embed_flat", flat);
    save("gen_expand", expanded);
    std::cout << "shape " << shape(input_ids) << " seq " << gather(shape(input_ids), GraphPrologue::c_one) << "\n";

    check_cuda(cudaStreamSynchronize(stream));
    std::printf("conformance ok\n");
    return 0;
}
