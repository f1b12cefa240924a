// Deferred.hpp - deferred evaluation of the eager API: element-wise calls and
// reductions on CUDA tensors record their work in the result's storage and
// run where a consumer needs the buffer, so unchanged generated code (a chain
// of separate operator calls) fuses into few kernels.  This is the
// reference's tape merge (MergeNodes, Node.hpp:189-224; ExecutionTape::Append
// / Optimize, ExecutionTape.hpp:41-102) carried out at run time behind the
// ordinary operators.
//
// A deferred element-wise result holds a chain (tadma_instr program over up
// to 6 operand views, TADMA_MAX_INPUTS) and a reduction result holds a
// reduce_chain call plus a post chain.  A new call whose accumulator operand
// is a deferred result of the same dims, read as its whole row-major buffer,
// copies that result's chain and appends its own instruction ("splices"): the
// intermediate never reaches HBM unless something else reads it.  Likewise a
// reduction of such a result becomes one tadma_b200_reduce_chain, and an
// element-wise call with immediate operands only on a deferred reduction
// result extends its post chain (tadma_b200_reduce_chain_post).  Every
// instruction keeps the rounding and the precision of the call it replaces,
// so results are the bits the eager calls produce (sums: the same fold order
// where the fused kernel is the same row kernel, else within the reduction
// tolerance).
//
// Synchronisation (every library call of the header API goes through it):
// * reading a buffer (Tensor::describe, host copies, scalar()) first enqueues
//   the work deferred into that buffer;
// * writing a buffer (in-place calls, copies into it, node kernels) first
//   enqueues that work and every deferred work that reads the buffer;
// * work nobody reads is dropped with its buffer.
// All of it runs on the stream that was current when the call was made.  An
// error of a deferred call is raised where the work is enqueued.  Raw access
// to `data.view` of a result bypasses this: call materialize() first.
// set_deferred(false) (or TADMA_DEFER=0 in the environment) makes every call
// launch at once, as the reference's separate nodes do.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cstdlib>
#include <initializer_list>
#include <cstring>
#include <memory>
#include <vector>

#include "Core.hpp"

namespace tadma {

namespace detail {

inline bool defer_default() {
    const char* e = std::getenv("TADMA_DEFER");
    return !(e && e[0] == '0');
}
inline thread_local bool defer_enabled = defer_default();

}  // namespace detail

// Deferred evaluation on (the default) or off for the calling thread.
inline void set_deferred(bool on) { detail::defer_enabled = on; }
inline bool deferred() { return detail::defer_enabled; }

namespace detail {

inline bool dtype_float(int d) { return d == TADMA_F32 || d == TADMA_F16 || d == TADMA_BF16 || d == TADMA_F64; }
inline bool dtype_wide(int d) { return d == TADMA_F64 || d == TADMA_I64; }
inline bool dtype_16(int d) { return d == TADMA_F16 || d == TADMA_BF16; }
inline bool op_transcendental(int op) {
    return (op >= TADMA_OP_EXP && op <= TADMA_OP_GELU && op != TADMA_OP_RELU) || op == TADMA_OP_POW;
}

// The precision tadma_b200_eltwise picks (TADMA_COMPUTE_AUTO) for the one-op
// call y = op(a[, b | imm][, c]) that the eager API makes (-1: no operand).
inline int eager_compute(int out_dt, int a_dt, int b_dt, int op, bool has_imm, double imm, int c_dt = -1) {
    bool all_int = !dtype_float(out_dt) && (a_dt < 0 || !dtype_float(a_dt));
    bool wide = dtype_wide(out_dt) || (a_dt >= 0 && dtype_wide(a_dt));
    for (int d : {b_dt, c_dt}) {
        if (d < 0) continue;
        all_int = all_int && !dtype_float(d);
        wide = wide || dtype_wide(d);
    }
    if (op_transcendental(op)) all_int = false;
    if (has_imm && imm != (double)(int64_t)imm) all_int = false;
    if (all_int) return TADMA_COMPUTE_I64;
    return wide ? TADMA_COMPUTE_F64 : TADMA_COMPUTE_F32;
}

inline bool same_view(const tadma_tensor& u, const tadma_tensor& t) {
    bool same = u.data == t.data && u.dtype == t.dtype && u.rank == t.rank;
    for (int d = 0; same && d < t.rank; d++) same = u.dims[d] == t.dims[d] && u.strides[d] == t.strides[d];
    return same;
}

inline bool same_dims(const tadma_tensor& u, const tadma_tensor& t) {
    bool same = u.rank == t.rank;
    for (int d = 0; same && d < t.rank; d++) same = u.dims[d] == t.dims[d];
    return same;
}

inline int64_t desc_numel(const tadma_tensor& t) {
    int64_t n = 1;
    for (int d = 0; d < t.rank; d++) n *= t.dims[d];
    return n;
}

// Row-major contiguous (extent-1 dims ignored).
inline bool desc_contiguous(const tadma_tensor& t) {
    int64_t expect = 1;
    for (int d = t.rank - 1; d >= 0; d--) {
        if (t.dims[d] != 1 && t.strides[d] != expect) return false;
        expect *= t.dims[d];
    }
    return true;
}

// `op` with its operands swapped: b (op) a == swapped(op)(a, b); -1 if none.
constexpr int swapped_op(int op) {
    switch (op) {
    case TADMA_OP_SUB: return TADMA_OP_RSUB;
    case TADMA_OP_DIV: return TADMA_OP_RDIV;
    case TADMA_OP_RSUB: return TADMA_OP_SUB;
    case TADMA_OP_RDIV: return TADMA_OP_DIV;
    case TADMA_OP_GT: return TADMA_OP_LT;
    case TADMA_OP_LT: return TADMA_OP_GT;
    case TADMA_OP_GE: return TADMA_OP_LE;
    case TADMA_OP_LE: return TADMA_OP_GE;
    case TADMA_OP_ADD: case TADMA_OP_MUL: case TADMA_OP_MAX: case TADMA_OP_MIN: case TADMA_OP_EQ: case TADMA_OP_NE:
    case TADMA_OP_AND: case TADMA_OP_OR: case TADMA_OP_XOR: case TADMA_OP_LAND: case TADMA_OP_LOR:
        return op;
    default: return -1;
    }
}

// One operand of deferred work: its view, a reference that keeps its buffer
// alive, and its control block (null for a non-owning view).
struct DOperand {
    tadma_tensor desc{};
    std::shared_ptr<const void> keep;
    StorageCtl* ctl = nullptr;
};

// Work deferred into one buffer.
struct Deferred {
    tadma_tensor out{};  // the result: the buffer's whole row-major view
    std::array<tadma_instr, TADMA_MAX_INSTR> prog{};
    std::array<DOperand, TADMA_MAX_INPUTS> ins{};
    int n_instr = 0, n_ins = 0;
    int compute = TADMA_COMPUTE_AUTO;
    bool reduce = false;  // a tadma_b200_reduce_chain_post call
    bool plain = false;   // a reduction of ins[0] alone: tadma_b200_reduce, as the eager call
    int red_op = 0, axis = 0;
    std::array<tadma_instr, TADMA_MAX_INSTR> post{};
    int n_post = 0;
    cudaStream_t stream = nullptr;
    bool done = false;
};

inline void run(Deferred& d);
inline int launch_compute(const Deferred& d);

// Reading a buffer: enqueue the work deferred into it.
inline void sync_read(StorageCtl* c) {
    if (!c || !c->pending) return;
    std::shared_ptr<Deferred> d = std::move(c->pending);
    c->pending.reset();
    if (!d->done) run(*d);
}

// Writing a buffer: enqueue its own deferred work and every deferred work
// that reads it.
inline void sync_write(StorageCtl* c);
// The same for a tensor (a lazy value has no storage of its own: nothing to do).
template <typename T>
void sync_write_of(const T& t) {
    if constexpr (requires { t.data.ctl; }) sync_write(t.data.ctl);
}
inline void sync_write(StorageCtl* c) {
    if (!c) return;
    sync_read(c);
    std::vector<std::weak_ptr<Deferred>> readers;
    readers.swap(c->readers);
    for (auto& w : readers)
        if (auto d = w.lock())
            if (!d->done) run(*d);
}

inline bool try_row_program(Deferred& d);

inline void run(Deferred& d) {
    if (d.done) return;
    if (!d.reduce && try_row_program(d)) return;
    d.done = true;  // before the operands' own work runs: no re-entry
    std::array<tadma_tensor, TADMA_MAX_INPUTS> ins{};
    for (int k = 0; k < d.n_ins; k++) {
        sync_read(d.ins[k].ctl);
        ins[k] = d.ins[k].desc;
    }
    if (d.plain) {
        check(tadma_b200_reduce(d.red_op, &ins[0], d.axis, TADMA_OP_COPY, &d.out, d.stream), "tadma reduce (deferred)");
    } else if (d.reduce) {
        check(tadma_b200_reduce_chain_post(d.red_op, ins.data(), d.n_ins, d.prog.data(), d.n_instr, d.post.data(),
                                           d.n_post, d.compute, d.axis, &d.out, d.stream),
              "tadma reduce (deferred)");
    } else {
        check(tadma_b200_eltwise(&d.out, ins.data(), d.n_ins, d.prog.data(), d.n_instr, launch_compute(d), d.stream),
              "tadma eltwise (deferred)");
    }
    // The kernel reads the operands in stream order; dropping the references
    // frees a buffer behind it (stream-ordered free).
    for (int k = 0; k < d.n_ins; k++) d.ins[k] = DOperand{};
}

// The deferred element-wise work of `c` whose result `v` is: the whole buffer,
// row-major, dims as `v` (nullptr if `c` holds none or `v` is another view).
inline Deferred* spliceable(StorageCtl* c, const tadma_tensor& v, bool need_same_dims) {
    if (!c || !c->pending || c->pending->done || c->pending->reduce) return nullptr;
    Deferred* p = c->pending.get();
    if (v.data != p->out.data || v.dtype != p->out.dtype || !desc_contiguous(v) ||
        desc_numel(v) != desc_numel(p->out))
        return nullptr;
    if (need_same_dims && !same_dims(v, p->out)) return nullptr;
    return p;
}

inline int find_operand(const Deferred& d, const tadma_tensor& t) {
    for (int k = 0; k < d.n_ins; k++)
        if (same_view(d.ins[k].desc, t)) return k;
    return -1;
}

// Index of operand `o` in `d`, added if new; -1 when `d` is full.
inline int add_operand(Deferred& d, const DOperand& o) {
    int k = find_operand(d, o.desc);
    if (k >= 0) return k;
    if (d.n_ins >= TADMA_MAX_INPUTS) return -1;
    d.ins[d.n_ins] = o;
    return d.n_ins++;
}

// Registers `d` as a reader of each operand buffer it holds.
inline void register_reader(const std::shared_ptr<Deferred>& d) {
    for (int k = 0; k < d->n_ins; k++) {
        StorageCtl* c = d->ins[k].ctl;
        if (!c) continue;
        auto& r = c->readers;
        // drop finished readers so the list stays short
        r.erase(std::remove_if(r.begin(), r.end(),
                               [](const std::weak_ptr<Deferred>& w) {
                                   auto p = w.lock();
                                   return !p || p->done;
                               }),
                r.end());
        r.push_back(d);
    }
}

// The fast-math bodies of tadma_b200_eltwise (an fp32 chain ending in a
// 16-bit store) are what the eager call uses for an instruction that rounds
// to 16 bits; a transcendental instruction that the eager call computed into
// an fp32 tensor needs the precise bodies.
inline int launch_compute(const Deferred& d) {
    if (d.compute != TADMA_COMPUTE_F32 || !dtype_16(d.out.dtype)) return d.compute;
    for (int i = 0; i < d.n_instr; i++)
        if (op_transcendental(d.prog[i].op) && !dtype_16(d.prog[i].round_dtype)) return TADMA_COMPUTE_F32_PRECISE;
    return d.compute;
}

}  // namespace detail

namespace detail {

// --------------------------------------------------------- deferring calls --

// The precision TADMA_COMPUTE_AUTO resolves to for out = prog(ins...) (the
// rule of tadma_b200_eltwise).
inline int auto_compute(int out_dt, const int* in_dts, int n_ins, const tadma_instr* prog, int n_instr) {
    bool all_int = !dtype_float(out_dt);
    bool wide = dtype_wide(out_dt);
    for (int k = 0; k < n_ins; k++) {
        if (dtype_float(in_dts[k])) all_int = false;
        if (dtype_wide(in_dts[k])) wide = true;
    }
    for (int i = 0; i < n_instr; i++) {
        if (op_transcendental(prog[i].op)) all_int = false;
        if ((prog[i].b == TADMA_SRC_IMM || prog[i].c == TADMA_SRC_IMM) && prog[i].imm != (double)(int64_t)prog[i].imm)
            all_int = false;
    }
    if (all_int) return TADMA_COMPUTE_I64;
    return wide ? TADMA_COMPUTE_F64 : TADMA_COMPUTE_F32;
}

template <typename T>
DOperand make_operand(const T& t) {
    DOperand o;
    o.desc = t.describe_raw();
    o.keep = std::make_shared<const T>(t);
    o.ctl = t.data.ctl;
    return o;
}

inline bool imm_only(const tadma_instr& I) {
    const bool b_ok = I.b == TADMA_SRC_IMM || I.b == TADMA_SRC_NONE;
    const bool c_ok = I.c == TADMA_SRC_IMM || I.c == TADMA_SRC_NONE;
    return b_ok && c_ok && I.op != TADMA_OP_WHERE;
}

// Appends the call's program to `d`, whose accumulator already holds the
// call's input 0: operand references k >= 1 map to `d`'s operands (added if
// new).  False (and `d` partly modified) when a limit is hit or the program
// names input 0 as an operand.
inline bool append_program(Deferred& d, const tadma_instr* prog, int n_instr, const DOperand* ops, int n_ops) {
    if (d.n_instr + n_instr > TADMA_MAX_INSTR) return false;
    int map[TADMA_MAX_INPUTS + 1];
    for (int k = 1; k < n_ops; k++) {
        map[k] = add_operand(d, ops[k]);
        if (map[k] < 0) return false;
    }
    for (int i = 0; i < n_instr; i++) {
        tadma_instr I = prog[i];
        for (int32_t* sel : {&I.b, &I.c}) {
            if (*sel == 0) return false;
            if (*sel > 0) *sel = map[*sel];
        }
        d.prog[d.n_instr++] = I;
    }
    return true;
}

// out = prog(inputs...) (one eager call, CUDA tensors): recorded in out's
// storage instead of launched, splicing a deferred accumulator input.
// Returns false when the call must run now (the caller launches it).
template <typename Out, typename... In>
bool defer_eltwise(const Out& out, std::initializer_list<tadma_instr> prog_list, const In&... inputs) {
    constexpr int n = (int)sizeof...(In);
    if (!defer_enabled || n == 0 || n > TADMA_MAX_INPUTS) return false;
    StorageCtl* oc = out.data.ctl;
    if (!oc) return false;
    const tadma_instr* prog = prog_list.begin();
    const int n_instr = (int)prog_list.size();
    const tadma_tensor o = out.describe_raw();
    const DOperand ops[n] = {make_operand(inputs)...};
    int dts[n];
    for (int k = 0; k < n; k++) dts[k] = ops[k].desc.dtype;
    const int cm = auto_compute(o.dtype, dts, n, prog, n_instr);
    auto has_live_readers = [](StorageCtl* c) {
        for (auto& w : c->readers)
            if (auto p = w.lock())
                if (!p->done) return true;
        return false;
    };

    if (ops[0].desc.data == o.data) {
        // In place (x = f(x, ...)): extend the buffer's own deferred work.
        if (!oc->pending || oc->pending->done || has_live_readers(oc)) return false;
        Deferred& p = *oc->pending;
        if (!desc_contiguous(o) || desc_numel(o) != desc_numel(p.out) || o.dtype != p.out.dtype) return false;
        if (p.compute != cm) return false;
        if (p.reduce) {
            if (p.plain || p.red_op == TADMA_REDUCE_ARGMAX || p.red_op == TADMA_REDUCE_ARGMIN) return false;
            if (p.n_post + n_instr + 1 > TADMA_MAX_INSTR) return false;
            for (int i = 0; i < n_instr; i++)
                if (!imm_only(prog[i])) return false;
            if (p.n_post == 0) {
                tadma_instr r{};
                r.op = TADMA_OP_COPY;
                r.b = r.c = TADMA_SRC_NONE;
                r.round_dtype = p.out.dtype;
                p.post[p.n_post++] = r;
            }
            for (int i = 0; i < n_instr; i++) p.post[p.n_post++] = prog[i];
            return true;
        }
        for (int k = 1; k < n; k++)
            if (!same_dims(ops[k].desc, p.out)) return false;
        Deferred ext = p;
        if (!append_program(ext, prog, n_instr, ops, n)) return false;
        p = ext;
        register_reader(oc->pending);
        return true;
    }

    // A fresh result: the only handle of a whole, unread buffer.
    if (oc->refs.load() != 1 || oc->pending || has_live_readers(oc) || !desc_contiguous(o)) return false;
    auto d = std::make_shared<Deferred>();
    bool built = false;
    StorageCtl* c0 = ops[0].ctl;
    if (c0 && c0->pending && !c0->pending->done && c0->pending->compute == cm && same_dims(ops[0].desc, o)) {
        const Deferred& q = *c0->pending;
        if (q.reduce) {
            // Immediate-operand steps on a reduction result: its post chain,
            // after a rounding of the reduced value to the result's own type
            // (what storing it would do).
            const bool arg = q.red_op == TADMA_REDUCE_ARGMAX || q.red_op == TADMA_REDUCE_ARGMIN;
            bool ok = !arg && !q.plain && q.n_post + n_instr + 1 <= TADMA_MAX_INSTR && desc_contiguous(ops[0].desc) &&
                      ops[0].desc.data == q.out.data && ops[0].desc.dtype == q.out.dtype &&
                      desc_numel(ops[0].desc) == desc_numel(q.out);
            for (int i = 0; i < n_instr && ok; i++) ok = imm_only(prog[i]);
            if (ok) {
                *d = q;
                d->out = o;
                if (d->n_post == 0) {
                    tadma_instr r{};
                    r.op = TADMA_OP_COPY;
                    r.b = r.c = TADMA_SRC_NONE;
                    r.round_dtype = q.out.dtype;
                    d->post[d->n_post++] = r;
                }
                for (int i = 0; i < n_instr; i++) d->post[d->n_post++] = prog[i];
                built = true;
            }
        } else if (spliceable(c0, ops[0].desc, true)) {
            *d = q;
            d->out = o;
            built = append_program(*d, prog, n_instr, ops, n);
        }
    }
    if (!built && n == 2 && n_instr == 1 && prog[0].b == 1 && prog[0].c == TADMA_SRC_NONE &&
        swapped_op(prog[0].op) >= 0 && same_dims(ops[1].desc, o)) {
        // b (op) a with b deferred: b becomes the accumulator.
        StorageCtl* c1 = ops[1].ctl;
        if (c1 && spliceable(c1, ops[1].desc, true) && c1->pending->compute == cm) {
            *d = *c1->pending;
            d->out = o;
            tadma_instr I = prog[0];
            I.op = swapped_op(I.op);
            const int k = add_operand(*d, ops[0]);
            if (k >= 0 && d->n_instr < TADMA_MAX_INSTR) {
                I.b = k;
                d->prog[d->n_instr++] = I;
                built = true;
            }
        }
    }
    if (!built) {
        // A chain of its own over the inputs (deferred inputs run first).
        *d = Deferred{};
        d->out = o;
        for (int k = 0; k < n; k++) d->ins[k] = ops[k];
        d->n_ins = n;
        for (int i = 0; i < n_instr; i++) d->prog[i] = prog[i];
        d->n_instr = n_instr;
    }
    d->out = o;
    d->compute = cm;
    d->stream = stream;
    d->done = false;
    oc->pending = d;
    register_reader(d);
    return true;
}

// out = reduce(t) (one eager reduction) over a deferred element-wise result
// t: one tadma_b200_reduce_chain_post over t's chain, itself deferred so
// that immediate-operand steps on the result become its post chain.  False
// when `t` holds no such chain (the caller reduces at once).
// Reduced extents from this length on may split across CTAs in the eager
// reduction (another fold order); those reductions are not deferred.
constexpr int64_t kDeferMaxAxis = 16384;

template <typename Out, typename T>
bool defer_reduce(int op, int axis, const Out& out, const T& t) {
    if (!defer_enabled) return false;
    StorageCtl* oc = out.data.ctl;
    StorageCtl* tc = t.data.ctl;
    const tadma_tensor i = t.describe_raw();
    if (!oc || !tc || oc->refs.load() != 1 || oc->pending) return false;
    if (i.dims[axis] >= kDeferMaxAxis) return false;
    Deferred* q = spliceable(tc, i, true);
    if (!q) return false;
    auto d = std::make_shared<Deferred>(*q);
    d->reduce = true;
    d->red_op = op;
    d->axis = axis;
    d->n_post = 0;
    d->out = out.describe_raw();
    d->stream = stream;
    d->done = false;
    oc->pending = d;
    register_reader(d);
    return true;
}

// out = reduce of t over its last axis (SUM, MEAN, MAX, MIN of a float
// tensor), t holding no chain to splice: deferred as the eager
// tadma_b200_reduce call, so that a row program can take it as a stage.
template <typename Out, typename T>
bool defer_plain_reduce(int op, int axis, const Out& out, const T& t) {
    if (!defer_enabled) return false;
    if (op != TADMA_REDUCE_SUM && op != TADMA_REDUCE_MEAN && op != TADMA_REDUCE_MAX && op != TADMA_REDUCE_MIN) return false;
    StorageCtl* oc = out.data.ctl;
    if (!oc || !t.data.ctl || oc->refs.load() != 1 || oc->pending) return false;
    const tadma_tensor i = t.describe_raw();
    if (axis != i.rank - 1 || i.dims[axis] >= kDeferMaxAxis) return false;
    if (i.dtype != TADMA_F32 && i.dtype != TADMA_F16 && i.dtype != TADMA_BF16) return false;
    auto d = std::make_shared<Deferred>();
    d->reduce = d->plain = true;
    d->red_op = op;
    d->axis = axis;
    d->ins[0] = make_operand(t);
    d->n_ins = 1;
    d->compute = TADMA_COMPUTE_F32;
    d->out = out.describe_raw();
    d->stream = stream;
    oc->pending = d;
    register_reader(d);
    return true;
}

// ------------------------------------------------------------- row program --
//
// An element-wise chain whose operands include deferred reductions over the
// last axis of rows of its own shape (a LayerNorm written out: mean, -, pow,
// mean, + eps, sqrt, /, *, +) runs as one tadma_b200_row_program: the
// reductions become its stages (their own deferred reductions first) and
// the chain its final program.  The row program gives the bits of the
// separate calls; grids it does not take (TADMA_ERR_UNSUPPORTED) run as
// before.

// A view of `t` over the {rows, cols} grid of `o`: a row operand (o's dims,
// contiguous rows), a column operand (leading dims 1) or a row scalar (last
// dim 1, leading dims o's with uniform row stride, or all 1).  False if none.
inline bool grid_view(const tadma_tensor& t, const tadma_tensor& o, int64_t rows, int64_t cols, tadma_tensor& v) {
    if (t.rank != o.rank) return false;
    const int last = o.rank - 1;
    bool lead_one = true, lead_same = true;
    for (int d = 0; d < last; d++) {
        if (t.dims[d] != 1 && t.strides[d] != 0) lead_one = false;
        if (t.dims[d] != o.dims[d]) lead_same = false;
    }
    // uniform row stride over the leading dims (row-major row index)
    auto row_stride = [&](int64_t& rs) {
        rs = 0;
        int64_t span = 1;
        bool first = true;
        for (int d = last - 1; d >= 0; d--) {
            if (o.dims[d] == 1) continue;
            if (first) {
                rs = t.strides[d];
                first = false;
            } else if (t.strides[d] != rs * span) {
                return false;
            }
            span *= o.dims[d];
        }
        return true;
    };
    v = tadma_tensor{};
    v.data = t.data;
    v.dtype = t.dtype;
    v.rank = 2;
    v.dims[0] = rows;
    v.dims[1] = cols;
    const bool vec = t.dims[last] == cols && (cols == 1 || t.strides[last] == 1);
    const bool scal = t.dims[last] == 1 || t.strides[last] == 0;
    int64_t rs = 0;
    if (vec && cols > 1) {
        if (lead_one) {
            v.dims[0] = 1;
            v.strides[0] = 0;
        } else if (lead_same && row_stride(rs) && rs == cols) {
            v.strides[0] = rs;
        } else {
            return false;
        }
        v.strides[1] = 1;
        return true;
    }
    if (scal) {
        v.dims[1] = 1;
        v.strides[1] = 0;
        if (lead_one) {
            v.dims[0] = 1;
            v.strides[0] = 0;
        } else if (lead_same && row_stride(rs)) {
            v.strides[0] = rs;
        } else {
            return false;
        }
        return true;
    }
    return false;
}

inline bool try_row_program(Deferred& d) {
    if (d.reduce || d.compute != TADMA_COMPUTE_F32 || d.n_ins < 1) return false;
    const tadma_tensor& o = d.out;
    if (o.rank < 1 || !desc_contiguous(o)) return false;
    const int last = o.rank - 1;
    const int64_t cols = o.dims[last];
    if (cols < 1) return false;
    const int64_t rows = desc_numel(o) / cols;
    if (rows < 1) return false;

    // The stages: deferred reductions among the operands, their own first.
    std::vector<std::shared_ptr<Deferred>> stages;
    auto stage_of = [&](const DOperand& op) -> std::shared_ptr<Deferred> {
        if (!op.ctl || !op.ctl->pending || op.ctl->pending->done || !op.ctl->pending->reduce) return nullptr;
        return op.ctl->pending;
    };
    bool ok = true;
    auto collect = [&](auto&& self, const Deferred& q, int depth) -> void {
        for (int k = 0; k < q.n_ins && ok; k++) {
            std::shared_ptr<Deferred> s = stage_of(q.ins[k]);
            if (!s) continue;
            if (std::find(stages.begin(), stages.end(), s) != stages.end()) continue;
            const int op = s->red_op;
            if (depth > TADMA_ROWPROG_MAX_STAGES || s->compute != TADMA_COMPUTE_F32 || s->axis != last ||
                !(op == TADMA_REDUCE_SUM || op == TADMA_REDUCE_MEAN || op == TADMA_REDUCE_MAX || op == TADMA_REDUCE_MIN) ||
                !desc_contiguous(s->out) || desc_numel(s->out) != rows) {
                ok = false;
                return;
            }
            // the reduced grid is o's: each operand broadcasts to o's dims
            for (int j = 0; j < s->n_ins && ok; j++) {
                const tadma_tensor& t = s->ins[j].desc;
                if (t.rank != o.rank) ok = false;
                for (int dd = 0; dd < t.rank && ok; dd++)
                    if (t.dims[dd] != o.dims[dd] && t.dims[dd] != 1) ok = false;
            }
            if (!ok) return;
            self(self, *s, depth + 1);
            stages.push_back(s);
        }
    };
    collect(collect, d, 0);
    if (!ok || stages.empty() || (int)stages.size() > TADMA_ROWPROG_MAX_STAGES) return false;

    // Operands: every view that is not a stage result, numbered first.
    tadma_row_program rp{};
    rp.rows = rows;
    rp.cols = cols;
    std::vector<StorageCtl*> leaf_ctl;
    auto number = [&](const DOperand& op) -> int {
        std::shared_ptr<Deferred> s = stage_of(op);
        if (s) {
            const int si = (int)(std::find(stages.begin(), stages.end(), s) - stages.begin());
            // the consumer reads the stage's whole buffer as one value per row
            tadma_tensor v;
            if (op.desc.data != s->out.data || !grid_view(op.desc, o, rows, cols, v) || v.dims[1] != 1 ||
                (rows > 1 && v.strides[0] != 1))
                return -1;
            return 1000 + si;  // resolved once the leaves are counted
        }
        tadma_tensor v;
        if (!grid_view(op.desc, o, rows, cols, v)) return -1;
        for (int k = 0; k < rp.n_ins; k++)
            if (rp.ins[k].data == v.data && rp.ins[k].dtype == v.dtype && rp.ins[k].dims[0] == v.dims[0] &&
                rp.ins[k].dims[1] == v.dims[1] && rp.ins[k].strides[0] == v.strides[0] && rp.ins[k].strides[1] == v.strides[1])
                return k;
        if (rp.n_ins == TADMA_MAX_INPUTS) return -1;
        rp.ins[rp.n_ins] = v;
        leaf_ctl.push_back(op.ctl);
        return rp.n_ins++;
    };
    // operand numbers of each stage's and of the final chain's inputs
    std::vector<std::array<int, TADMA_MAX_INPUTS>> smap(stages.size());
    for (size_t si = 0; si < stages.size(); si++)
        for (int k = 0; k < stages[si]->n_ins; k++)
            if ((smap[si][k] = number(stages[si]->ins[k])) < 0) return false;
    std::array<int, TADMA_MAX_INPUTS> dmap{};
    for (int k = 0; k < d.n_ins; k++)
        if ((dmap[k] = number(d.ins[k])) < 0) return false;
    auto resolve = [&](int n) { return n >= 1000 ? rp.n_ins + (n - 1000) : n; };
    auto remap = [&](const tadma_instr* prog, int n_instr, const std::array<int, TADMA_MAX_INPUTS>& map, tadma_instr* dst) {
        for (int i = 0; i < n_instr; i++) {
            tadma_instr I = prog[i];
            if (I.b >= 0) I.b = resolve(map[I.b]);
            if (I.c >= 0) I.c = resolve(map[I.c]);
            dst[i] = I;
        }
    };
    rp.n_stages = (int32_t)stages.size();
    for (size_t si = 0; si < stages.size(); si++) {
        const Deferred& s = *stages[si];
        tadma_row_stage& st = rp.stages[si];
        st.op = s.red_op;
        st.n_instr = s.n_instr;
        st.n_post = s.n_post;
        st.acc = resolve(smap[si][0]);
        remap(s.prog.data(), s.n_instr, smap[si], st.prog);
        for (int i = 0; i < s.n_post; i++) st.post[i] = s.post[i];
        st.out = tadma_tensor{};
        st.out.data = s.out.data;
        st.out.dtype = s.out.dtype;
        st.out.rank = 1;
        st.out.dims[0] = rows;
        st.out.strides[0] = 1;
    }
    rp.n_instr = d.n_instr;
    remap(d.prog.data(), d.n_instr, dmap, rp.prog);
    rp.acc = resolve(dmap[0]);
    rp.compute = launch_compute(d);
    rp.out = tadma_tensor{};
    rp.out.data = o.data;
    rp.out.dtype = o.dtype;
    rp.out.rank = 2;
    rp.out.dims[0] = rows;
    rp.out.dims[1] = cols;
    rp.out.strides[0] = cols;
    rp.out.strides[1] = 1;

    // the inputs' own deferred work first
    for (StorageCtl* c : leaf_ctl) sync_read(c);
    const int rc = tadma_b200_row_program(&rp, d.stream);
    if (rc == TADMA_ERR_UNSUPPORTED) return false;
    check(rc, "tadma row program (deferred)");
    d.done = true;
    for (auto& s : stages) {
        s->done = true;
        for (int k = 0; k < s->n_ins; k++) s->ins[k] = DOperand{};
    }
    for (int k = 0; k < d.n_ins; k++) d.ins[k] = DOperand{};
    return true;
}

}  // namespace detail

}  // namespace tadma
