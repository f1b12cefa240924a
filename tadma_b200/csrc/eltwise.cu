// eltwise.cu - fused element-wise / broadcast engine (sm_100a).
//
// Replaces the reference's lazy-node executor: EltwiseNode / CombineToNode /
// CombineNode / InplaceNode (Kernels.hpp:16-53) run through CUDAHIPExecutor
// (Node.hpp:25-48): one scalar element per thread, 512-thread blocks, a 32-bit
// index and an int64 div/mod per dimension per element.  MergeNodes
// (Node.hpp:189-224) composes node lambdas into one kernel; here a fused
// chain is a short instruction list (tadma_instr) evaluated in registers.
//
// Design:
// * the joint layout of out and inputs is folded (layout.hpp); typical
//   launches become rank 1 (streaming) or rank 2 (row broadcast);
// * vector path: each thread step handles V = 8 consecutive elements with
//   16-byte loads/stores (2 x 16 B for fp32, 1 x 16 B for 16-bit types); an
//   operand whose innermost stride is 0 is loaded once and splatted;
//   operands with no broadcast stream through with evict-first hints;
// * one contiguous chunk per CTA (U = 2 vector steps per thread, 1 with 3-4
//   operands, loaded before any compute) and as many CTAs as chunks, so the
//   block scheduler balances the SMs;
// * any other layout takes the scalar path (SU elements per thread, DivMod
//   index decomposition, still 64-bit safe);
// * the chain is uniform across the grid (kernel parameters), so the
//   per-instruction switch is a uniform branch amortised over 8 elements.
#include "eltwise_impl.cuh"

namespace tadma_b200 {

int blocks_per_sm(const void* fn) {
    static std::mutex mu;
    static std::unordered_map<const void*, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(fn);
    if (it != cache.end()) return it->second;
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, THREADS, 0) != cudaSuccess || nb <= 0) nb = 1;
    cache[fn] = nb;
    return nb;
}

namespace {

// Recognises [MUL imm]? [ADD ins[1]]? [GELU | RELU | SIGMOID | TANH]? in fp32
// compute with only no-op roundings (fp32 / fp64): act(x * s + b).
struct AffineMatch {
    bool ok = false, mul = false, add = false;
    int act = ACT_NONE;
    float scale = 1.0f;
};

AffineMatch match_affine(const tadma_instr* prog, int n_instr, int n_ins) {
    AffineMatch m;
    auto noop_round = [](int rd) { return rd < 0 || rd == TADMA_F32 || rd == TADMA_F64; };
    int i = 0;
    if (i < n_instr && prog[i].op == TADMA_OP_MUL && prog[i].b == TADMA_SRC_IMM && noop_round(prog[i].round_dtype)) {
        m.mul = true;
        m.scale = (float)prog[i].imm;
        i++;
    }
    if (i < n_instr && prog[i].op == TADMA_OP_ADD && prog[i].b == 1 && noop_round(prog[i].round_dtype)) {
        m.add = true;
        i++;
    }
    if (i < n_instr && noop_round(prog[i].round_dtype)) {
        switch (prog[i].op) {
        case TADMA_OP_GELU: m.act = ACT_GELU; i++; break;
        case TADMA_OP_RELU: m.act = ACT_RELU; i++; break;
        case TADMA_OP_SIGMOID: m.act = ACT_SIGMOID; i++; break;
        case TADMA_OP_TANH: m.act = ACT_TANH; i++; break;
        default: break;
        }
    }
    m.ok = i == n_instr && n_instr > 0 && n_ins == (m.add ? 2 : 1);
    return m;
}

bool is_transcendental(int op) { return op >= TADMA_OP_EXP && op <= TADMA_OP_GELU && op != TADMA_OP_RELU; }

// A chain of the row-operand reduction's form: [op1 m]? [unary]? [pow 2]?
// over ins[0], with m = ins[1] broadcast along the reduced axis (one value
// per output row) or an immediate, and only no-op roundings (fp32 compute).
struct RowOpMatch {
    bool ok = false;
    int op1 = TADMA_OP_COPY, pre = TADMA_OP_COPY, square = 0;
    const tadma_tensor* rop = nullptr;
    double imm1 = 0.0;
};

RowOpMatch match_rowop(const tadma_instr* prog, int n_instr, const tadma_tensor* ins, int n_ins, int ax) {
    RowOpMatch m;
    auto noop_round = [](int rd) { return rd < 0 || rd == TADMA_F32 || rd == TADMA_F64; };
    auto binop = [](int op) {
        return op == TADMA_OP_ADD || op == TADMA_OP_SUB || op == TADMA_OP_MUL || op == TADMA_OP_DIV ||
               op == TADMA_OP_RSUB || op == TADMA_OP_RDIV || op == TADMA_OP_MAX || op == TADMA_OP_MIN;
    };
    int i = 0;
    if (i < n_instr && binop(prog[i].op) && prog[i].c == TADMA_SRC_NONE && noop_round(prog[i].round_dtype)) {
        if (prog[i].b == TADMA_SRC_IMM && n_ins == 1) {
            m.op1 = prog[i].op;
            m.imm1 = prog[i].imm;
            i++;
        } else if (prog[i].b == 1 && n_ins == 2 && (ins[1].dims[ax] == 1 || ins[1].strides[ax] == 0)) {
            m.op1 = prog[i].op;
            m.rop = &ins[1];
            i++;
        }
    }
    auto is_pow2 = [&](int k) {
        return prog[k].op == TADMA_OP_POW && prog[k].b == TADMA_SRC_IMM && prog[k].imm == 2.0 && noop_round(prog[k].round_dtype);
    };
    if (i < n_instr && prog[i].op > TADMA_OP_COPY && prog[i].op < 32 && prog[i].op != TADMA_OP_NOT &&
        noop_round(prog[i].round_dtype)) {
        m.pre = prog[i].op;
        i++;
    }
    if (i < n_instr && is_pow2(i)) {
        m.square = 1;
        i++;
    }
    m.ok = i == n_instr && (n_ins == 1 || m.rop != nullptr);
    return m;
}

bool valid_op(int op) {
    return (op >= 0 && op <= TADMA_OP_NOT) || (op >= TADMA_OP_ADD && op <= TADMA_OP_LOR) || op == TADMA_OP_WHERE;
}

}  // namespace


// Same rule as the oracle: integer-only chains compute in int64, anything
// touching f64/i64 in f64, the rest in f32.
int resolve_compute(const tadma_tensor* out, const tadma_tensor* ins, int n_ins, const tadma_instr* prog, int n_instr,
                    int compute) {
    if (compute != TADMA_COMPUTE_AUTO) return compute;
    bool all_int = !dtype_is_float(out->dtype);
    bool any_wide = out->dtype == TADMA_F64 || out->dtype == TADMA_I64;
    for (int k = 0; k < n_ins; k++) {
        if (dtype_is_float(ins[k].dtype)) all_int = false;
        if (ins[k].dtype == TADMA_F64 || ins[k].dtype == TADMA_I64) any_wide = true;
    }
    for (int i = 0; i < n_instr; i++) {
        if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW) all_int = false;
        if ((prog[i].b == TADMA_SRC_IMM || prog[i].c == TADMA_SRC_IMM) && prog[i].imm != (double)(int64_t)prog[i].imm)
            all_int = false;
    }
    if (all_int) return TADMA_COMPUTE_I64;
    return any_wide ? TADMA_COMPUTE_F64 : TADMA_COMPUTE_F32;
}

}  // namespace tadma_b200

using namespace tadma_b200;

extern "C" int tadma_b200_eltwise(const tadma_tensor* out, const tadma_tensor* ins, int32_t n_ins,
                                  const tadma_instr* prog, int32_t n_instr, int32_t compute, void* stream) {
    std::string err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (n_ins < 0 || n_ins > TADMA_MAX_INPUTS) return fail(TADMA_ERR_INVALID, "n_ins out of range [0, 6]");
    if (n_instr < 0 || n_instr > TADMA_MAX_INSTR) return fail(TADMA_ERR_INVALID, "n_instr out of range [0, 16]");
    if (n_ins > 0 && !ins) return fail(TADMA_ERR_INVALID, "ins is NULL");
    if (n_instr > 0 && !prog) return fail(TADMA_ERR_INVALID, "prog is NULL");
    for (int k = 0; k < n_ins; k++) {
        err = check_tensor(&ins[k], "ins[k]");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (ins[k].rank != out->rank) return fail(TADMA_ERR_INVALID, "ins[k] rank differs from out rank");
        for (int d = 0; d < out->rank; d++)
            if (ins[k].dims[d] != out->dims[d] && ins[k].dims[d] != 1)
                return fail(TADMA_ERR_INVALID, "ins[k] dims not broadcastable to out dims");
    }
    for (int i = 0; i < n_instr; i++) {
        const tadma_instr& I = prog[i];
        if (!valid_op(I.op)) return fail(TADMA_ERR_INVALID, "unknown op code");
        bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
        if (needs_b && !(I.b == TADMA_SRC_IMM || (I.b >= 0 && I.b < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector b out of range");
        if (I.op == TADMA_OP_WHERE && !(I.c == TADMA_SRC_IMM || (I.c >= 0 && I.c < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector c out of range");
        if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return fail(TADMA_ERR_INVALID, "bad round_dtype");
    }
    const bool precise = compute == TADMA_COMPUTE_F32_PRECISE;
    int cm = precise ? TADMA_COMPUTE_F32 : resolve_compute(out, ins, n_ins, prog, n_instr, compute);
    if (cm < TADMA_COMPUTE_F32 || cm > TADMA_COMPUTE_I64) return fail(TADMA_ERR_INVALID, "bad compute mode");
    if (cm == TADMA_COMPUTE_I64)
        for (int i = 0; i < n_instr; i++)
            if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW)
                return fail(TADMA_ERR_UNSUPPORTED, "transcendental op in int64 compute");
    const int64_t n = numel(out);
    if (n == 0) return TADMA_OK;

    // Joint fold of out + inputs.
    int64_t strides[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    for (int d = 0; d < out->rank; d++) {
        strides[0][d] = out->strides[d];
        for (int k = 0; k < n_ins; k++) strides[1 + k][d] = (ins[k].dims[d] == 1) ? 0 : ins[k].strides[d];
    }
    Folded f = fold(out->rank, out->dims, strides, 1 + n_ins);

    ChainParams p{};
    p.rank = f.rank;
    p.n_instr = n_instr;
    p.out_dtype = out->dtype;
    p.out = (char*)out->data;
    for (int d = 0; d < f.rank; d++) {
        p.dims[d] = f.dims[d];
        p.out_stride[d] = f.strides[0][d];
    }
    for (int k = 0; k < n_ins; k++) {
        Operand& o = p.in[k];
        o.base = (const char*)ins[k].data;
        o.dtype = ins[k].dtype;
        o.streaming = 1;
        for (int d = 0; d < f.rank; d++) {
            o.stride[d] = f.strides[1 + k][d];
            if (o.stride[d] == 0 && f.dims[d] > 1) o.streaming = 0;
        }
        if (ins[k].data == out->data) o.streaming = 0;  // in-place: keep coherent loads
    }
    for (int i = 0; i < n_instr; i++) p.prog[i] = prog[i];

    // Vector-path eligibility.
    const int last = f.rank - 1;
    const int64_t inner = f.dims[last];
    auto aligned = [&](const void* ptr, int dt, const int64_t* st) {
        int64_t a = 8 * dtype_size(dt);
        if (a > 16) a = 16;
        if ((uintptr_t)ptr % (uintptr_t)a) return false;
        for (int d = 0; d < last; d++)
            if ((st[d] * dtype_size(dt)) % a) return false;
        return true;
    };
    bool vec = f.strides[0][last] == 1 && aligned(out->data, out->dtype, f.strides[0]);
    for (int k = 0; k < n_ins && vec; k++) {
        int64_t s = f.strides[1 + k][last];
        if (s == 1) vec = aligned(ins[k].data, ins[k].dtype, f.strides[1 + k]);
        else if (s == 0) p.in[k].inner_bcast = 1;
        else vec = false;
    }
    if (f.rank > 1 && inner % V) vec = false;
    if (n < V) vec = false;
    // Both paths decompose ELEMENT indices; a vector (V elements, inner % V
    // == 0 when rank > 1) never straddles a row.
    for (int d = 1; d < f.rank; d++) p.dm[d] = DivMod((uint64_t)f.dims[d]);
    p.idx32 = (uint64_t)n < 0xffffffffull ? 1 : 0;
    if (p.idx32) {
        // Largest offset of the output and of each input, with non-negative
        // strides only: below 2^31 everywhere allows 32-bit offset sums.
        bool small = true;
        for (int k = 0; k <= n_ins && small; k++) {
            int64_t top = 0;
            for (int d = 0; d < f.rank && small; d++) {
                const int64_t st = f.strides[k][d];
                if (st < 0 || st > 0x7fffffff) small = false;
                else top += (f.dims[d] - 1) * st;
                if (top > 0x7fffffff) small = false;
            }
        }
        if (small) p.idx32 = 2;
    }

    // Fast math (SFU exp / reciprocal) when an fp32 chain ends in a 16-bit
    // store and every intermediate rounding is to fp32 or coarser: the
    // approximation error is far below the output's half-ulp.
    bool fast = !precise && cm == TADMA_COMPUTE_F32 && (out->dtype == TADMA_F16 || out->dtype == TADMA_BF16);
    for (int i = 0; i < n_instr && fast; i++) {
        int rd = prog[i].round_dtype;
        if (!(rd < 0 || rd == TADMA_F32 || rd == TADMA_F16 || rd == TADMA_BF16)) fast = false;
    }
    cudaStream_t s = (cudaStream_t)stream;
    // Narrow operands (fp32 compute): the raw-word kernel keeps more loads in flight.
    bool narrow = vec && cm == TADMA_COMPUTE_F32;
    for (int k = 0; k < n_ins && narrow; k++) {
        const int es = dtype_size(ins[k].dtype);
        narrow = p.in[k].inner_bcast ? (es <= 4 && ins[k].dtype != TADMA_F64 && ins[k].dtype != TADMA_I64) : es <= 2;
    }
    auto go = [&](const ChainParams& pp, bool v, int64_t work) {
        switch (cm) {
        case TADMA_COMPUTE_F32: return launch_interp_f32(n_ins, fast, pp, v, work, s, narrow);
        case TADMA_COMPUTE_F64: return launch_interp_f64(n_ins, pp, v, work, s);
        default: return launch_interp_i64(n_ins, pp, v, work, s);
        }
    };
    if (!vec) {
        // A single input whose contiguous dim differs from the output's: tiled transpose.
        int dt_in = -1;
        if (n_ins == 1 && cm == TADMA_COMPUTE_F32 && f.rank >= 2 && f.strides[0][last] == 1 &&
            f.strides[1][last] != 1 && f.strides[1][last] != 0 && ins[0].data != out->data) {
            for (int d = 0; d < last; d++)
                if (f.strides[1][d] == 1) dt_in = d;
        }
        if (dt_in >= 0 && (f.dims[dt_in] + 31) / 32 <= 65535 && (f.dims[last] + 31) / 32 <= 0x7fffffff) {
            TransposeParams tp{};
            tp.in = (const char*)ins[0].data;
            tp.out = (char*)out->data;
            tp.in_dtype = ins[0].dtype;
            tp.out_dtype = out->dtype;
            tp.n_i = f.dims[dt_in];
            tp.n_j = f.dims[last];
            tp.in_sj = f.strides[1][last];
            tp.out_si = f.strides[0][dt_in];
            tp.nbatch = 1;
            for (int d = 0; d < last; d++) {
                if (d == dt_in) continue;
                tp.bdm[tp.nb] = DivMod((uint64_t)f.dims[d]);
                tp.b_in[tp.nb] = f.strides[1][d];
                tp.b_out[tp.nb] = f.strides[0][d];
                tp.nbatch *= f.dims[d];
                tp.nb++;
            }
            tp.chain = p;
            return launch_transpose(fast, tp, s);
        }
        p.start = 0;
        p.n = n;
        return go(p, false, n);
    }
    // Vector path: vector vi covers elements [vi * V, vi * V + V); a rank-1
    // tail of n % V elements goes to the scalar kernel afterwards.
    const int64_t nvec = n / V;
    ChainParams pv = p;
    pv.n = nvec;
    int rc;
    AffineMatch am = cm == TADMA_COMPUTE_F32 ? match_affine(prog, n_instr, n_ins) : AffineMatch{};
    const bool fdt = out->dtype == TADMA_F32 || out->dtype == TADMA_F16 || out->dtype == TADMA_BF16;
    const bool rows_ok = am.ok && am.add && f.rank == 2 && fdt && ins[0].dtype == ins[1].dtype &&
                         (ins[0].dtype == TADMA_F32 || ins[0].dtype == TADMA_F16 || ins[0].dtype == TADMA_BF16) &&
                         (out->dtype == ins[0].dtype || out->dtype == TADMA_F32) && f.strides[2][0] == 0 &&
                         f.strides[2][1] == 1 && f.strides[1][1] == 1 && f.strides[0][1] == 1 && !p.in[1].inner_bcast &&
                         !(precise && am.act != ACT_NONE);  // the row kernel's 16-bit activations are the fast bodies
    auto fdt3 = [](int dt) { return dt == TADMA_F32 || dt == TADMA_F16 || dt == TADMA_BF16; };
    // One float dtype over every operand: the typed kernels.  Single
    // instructions (typed1) take one or two streaming operands; chains take
    // 1-6 operands, innermost broadcasts included, on the pre-decoded program.
    bool one_dt = cm == TADMA_COMPUTE_F32 && n_ins >= 1 && fdt3(out->dtype);
    for (int k = 0; k < n_ins && one_dt; k++) one_dt = ins[k].dtype == ins[0].dtype && fdt3(ins[k].dtype);
    bool typed_ok = one_dt && (n_ins == 1 || n_ins == 2);
    for (int k = 0; k < n_ins && typed_ok; k++) typed_ok = !p.in[k].inner_bcast;
    // Typed chains: vector operands first, then the (at most two) operands
    // broadcast along the innermost dim, which the kernel keeps as scalars.
    ChainParams pt;
    int n_vec = 0, n_scal = 0;
    bool chain_ok = one_dt;
    if (chain_ok) {
        int slot_of[TADMA_MAX_INPUTS];
        for (int k = 0; k < n_ins; k++)
            if (!p.in[k].inner_bcast) slot_of[k] = n_vec++;
        for (int k = 0; k < n_ins; k++)
            if (p.in[k].inner_bcast) slot_of[k] = n_vec + n_scal++;
        chain_ok = n_vec >= 1 && n_scal <= 2;
        if (chain_ok) {
            pt = pv;
            for (int k = 0; k < n_ins; k++) pt.in[slot_of[k]] = pv.in[k];
            chain_ok = decode_fprog(prog, n_instr, n_ins, pt.fp, slot_of);
        }
    }
    // One instruction (or none: a cast) whose rounding is a no-op before the store.
    int op1 = -1;
    bool imm1 = false;
    if (typed_ok && n_instr <= 1) {
        const tadma_instr* I = n_instr == 1 ? &prog[0] : nullptr;
        const int rd = I ? I->round_dtype : -1;
        const bool round_ok = rd < 0 || rd == TADMA_F32 || rd == out->dtype;
        if (!I) {
            if (n_ins == 1) op1 = TADMA_OP_COPY;
        } else if (round_ok && I->op == TADMA_OP_COPY && I->b != TADMA_SRC_IMM && n_ins == 1) {
            op1 = TADMA_OP_COPY;
        } else if (round_ok && ins[0].dtype == out->dtype && I->c == TADMA_SRC_NONE &&
                   (I->op == TADMA_OP_ADD || I->op == TADMA_OP_SUB || I->op == TADMA_OP_MUL || I->op == TADMA_OP_DIV ||
                    I->op == TADMA_OP_RSUB || I->op == TADMA_OP_RDIV || I->op == TADMA_OP_MAX || I->op == TADMA_OP_MIN)) {
            if (I->b == TADMA_SRC_IMM && n_ins == 1) {
                op1 = I->op;
                imm1 = true;
            } else if (I->b == 1 && n_ins == 2) {
                op1 = I->op;
            }
        }
    }
    // Comparisons into bool and where(bool / u8, T, T) -> T, one instruction.
    int cmp_op = -1;
    bool cmp_imm = false, where_ok = false;
    if (n_instr == 1 && cm == TADMA_COMPUTE_F32) {
        const tadma_instr& I = prog[0];
        const int rd = I.round_dtype;
        bool no_bcast = true;
        for (int k = 0; k < n_ins; k++) no_bcast = no_bcast && !p.in[k].inner_bcast;
        if (no_bcast && out->dtype == TADMA_BOOL && (rd < 0 || rd == TADMA_BOOL || rd == TADMA_F32) &&
            I.op >= TADMA_OP_EQ && I.op <= TADMA_OP_GE && I.c == TADMA_SRC_NONE && fdt3(ins[0].dtype)) {
            if (I.b == TADMA_SRC_IMM && n_ins == 1) {
                cmp_op = I.op;
                cmp_imm = true;
            } else if (I.b == 1 && n_ins == 2 && ins[1].dtype == ins[0].dtype) {
                cmp_op = I.op;
            }
        }
        where_ok = no_bcast && I.op == TADMA_OP_WHERE && I.b == 1 && I.c == 2 && n_ins == 3 &&
                   (ins[0].dtype == TADMA_BOOL || ins[0].dtype == TADMA_U8) && fdt3(out->dtype) &&
                   ins[1].dtype == out->dtype && ins[2].dtype == out->dtype &&
                   (rd < 0 || rd == TADMA_F32 || rd == out->dtype);
    }
    // First match wins: the row-broadcast affine kernel, the typed single-op
    // kernels, compile-time affine programs, then the interpreted kernels.
    if (rows_ok) {
        // vec eligibility (checked above) already guarantees 16-byte alignment of
        // every row start and inner % 8 == 0.
        AffineRowsParams ap{};
        ap.x = (const char*)ins[0].data;
        ap.bias = (const char*)ins[1].data;
        ap.out = (char*)out->data;
        ap.rows = f.dims[0];
        ap.ncv = f.dims[1] / V;
        ap.x_rs = f.strides[1][0];
        ap.out_rs = f.strides[0][0];
        ap.scale = am.mul ? am.scale : 1.0f;
        rc = launch_rows(ins[0].dtype, out->dtype, am.act, ap, s);
    } else if (cmp_op >= 0) {
        rc = launch_cmp(ins[0].dtype, cmp_op, cmp_imm, pv, nvec, s);
    } else if (where_ok) {
        rc = launch_where(out->dtype, pv, nvec, s);
    } else if (op1 >= 0) {
        rc = launch_typed1(ins[0].dtype, out->dtype, op1, imm1, pv, nvec, s);
    } else if (am.ok) {
        pv.scale = am.scale;
        rc = launch_affine(am.act, fast, am.mul, am.add, pv, nvec, s, narrow);
    } else if (chain_ok) {
        rc = launch_typed(ins[0].dtype, out->dtype, n_vec, n_scal, fast, pt, nvec, s);
    } else {
        rc = go(pv, true, nvec);
    }
    if (rc != TADMA_OK) return rc;
    if (nvec * V < n) {
        p.start = nvec * V;
        p.n = n;
        return go(p, false, n - nvec * V);
    }
    return TADMA_OK;
}

static int reduce_chain_impl(int32_t op, const tadma_tensor* ins, int32_t n_ins, const tadma_instr* prog,
                             int32_t n_instr, const tadma_instr* post, int32_t n_post, int32_t compute, int32_t axis,
                             const tadma_tensor* out, void* stream) {
    std::string err = check_tensor(out, "out");
    if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
    if (n_ins < 1 || n_ins > TADMA_MAX_INPUTS) return fail(TADMA_ERR_INVALID, "n_ins out of range [1, 6]");
    if (n_instr < 0 || n_instr > TADMA_MAX_INSTR) return fail(TADMA_ERR_INVALID, "n_instr out of range [0, 16]");
    if (!ins) return fail(TADMA_ERR_INVALID, "ins is NULL");
    if (n_instr > 0 && !prog) return fail(TADMA_ERR_INVALID, "prog is NULL");
    if (op < TADMA_REDUCE_SUM || op > TADMA_REDUCE_RMS) return fail(TADMA_ERR_INVALID, "unknown reduce op");
    const int rank = ins[0].rank;
    if (rank < 1) return fail(TADMA_ERR_INVALID, "ins must have rank >= 1");
    int64_t S[TADMA_MAX_RANK];
    for (int d = 0; d < rank; d++) S[d] = 1;
    for (int k = 0; k < n_ins; k++) {
        err = check_tensor(&ins[k], "ins[k]");
        if (!err.empty()) return fail(TADMA_ERR_INVALID, err);
        if (ins[k].rank != rank) return fail(TADMA_ERR_INVALID, "ins must share one rank");
        for (int d = 0; d < rank; d++) {
            if (ins[k].dims[d] == 1) continue;
            if (S[d] != 1 && S[d] != ins[k].dims[d]) return fail(TADMA_ERR_INVALID, "ins dims do not broadcast");
            S[d] = ins[k].dims[d];
        }
    }
    for (int i = 0; i < n_instr; i++) {
        const tadma_instr& I = prog[i];
        if (!valid_op(I.op)) return fail(TADMA_ERR_INVALID, "unknown op code");
        bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
        if (needs_b && !(I.b == TADMA_SRC_IMM || (I.b >= 0 && I.b < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector b out of range");
        if (I.op == TADMA_OP_WHERE && !(I.c == TADMA_SRC_IMM || (I.c >= 0 && I.c < n_ins)))
            return fail(TADMA_ERR_INVALID, "operand selector c out of range");
        if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return fail(TADMA_ERR_INVALID, "bad round_dtype");
    }
    if (n_post < 0 || n_post > TADMA_MAX_INSTR) return fail(TADMA_ERR_INVALID, "n_post out of range [0, 16]");
    if (n_post > 0 && !post) return fail(TADMA_ERR_INVALID, "post is NULL");
    for (int i = 0; i < n_post; i++) {
        const tadma_instr& I = post[i];
        if (!valid_op(I.op)) return fail(TADMA_ERR_INVALID, "unknown op code in post");
        if (I.op == TADMA_OP_WHERE) return fail(TADMA_ERR_INVALID, "post: WHERE needs tensor operands");
        const bool needs_b = I.op >= 32 || (I.op == TADMA_OP_COPY && I.b == TADMA_SRC_IMM);
        if (needs_b && I.b != TADMA_SRC_IMM) return fail(TADMA_ERR_INVALID, "post: operands must be immediates");
        if (I.round_dtype >= 0 && dtype_size(I.round_dtype) == 0) return fail(TADMA_ERR_INVALID, "bad round_dtype in post");
    }
    const int ax = axis < 0 ? axis + rank : axis;
    if (ax < 0 || ax >= rank) return fail(TADMA_ERR_INVALID, "axis out of range");
    const bool keep = out->rank == rank;
    if (!keep && out->rank != rank - 1) return fail(TADMA_ERR_INVALID, "out rank must be rank or rank - 1");
    for (int d = 0, k = 0; d < rank; d++) {
        if (d == ax) {
            if (keep && out->dims[k++] != 1) return fail(TADMA_ERR_INVALID, "out dims[axis] must be 1");
            continue;
        }
        if (out->dims[k++] != S[d]) return fail(TADMA_ERR_INVALID, "out dims do not match the reduced dims");
    }
    const bool arg = op == TADMA_REDUCE_ARGMAX || op == TADMA_REDUCE_ARGMIN;
    if (arg && out->dtype != TADMA_I64 && out->dtype != TADMA_I32)
        return fail(TADMA_ERR_INVALID, "argmax/argmin output must be int64 or int32");
    if (arg && n_post > 0) return fail(TADMA_ERR_INVALID, "argmax/argmin take no post chain");
    // The chain's natural result type decides the compute type, as for a
    // materialised chain (ins[0]'s dtype standing in for the temporary's).
    tadma_tensor chain_out = ins[0];
    if (compute == TADMA_COMPUTE_F32_PRECISE) compute = TADMA_COMPUTE_F32;  // the reduction has no fast-math bodies
    int cm = resolve_compute(&chain_out, ins, n_ins, prog, n_instr, compute);
    if (cm < TADMA_COMPUTE_F32 || cm > TADMA_COMPUTE_I64) return fail(TADMA_ERR_INVALID, "bad compute mode");
    if (cm == TADMA_COMPUTE_I64)
        for (int i = 0; i < n_instr; i++)
            if (is_transcendental(prog[i].op) || prog[i].op == TADMA_OP_POW)
                return fail(TADMA_ERR_UNSUPPORTED, "transcendental op in int64 compute");
    const int64_t R = S[ax];
    if (R == 0 && op != TADMA_REDUCE_SUM && op != TADMA_REDUCE_SUMSQ)
        return fail(TADMA_ERR_INVALID, "empty reduction has no identity for this op");
    if (numel(out) == 0) return TADMA_OK;

    if (cm == TADMA_COMPUTE_F32) {
        // The row-operand form runs on the reduction engine's row kernel.
        RowOpMatch rm = match_rowop(prog, n_instr, ins, n_ins, ax);
        const bool op_sq = op == TADMA_REDUCE_SUMSQ || op == TADMA_REDUCE_RMS;
        if (rm.ok && !(rm.square && op_sq)) {
            int rc = reduce_rowop(op, S, rank, ax, &ins[0], rm.op1, rm.rop, rm.imm1, rm.pre, rm.square || op_sq, post,
                                  n_post, out, (cudaStream_t)stream);
            if (rc != TADMA_ERR_UNSUPPORTED) return rc;
        }
    }

    ChainReduceParams p{};
    p.pc.n = n_post;
    for (int i = 0; i < n_post; i++) p.pc.prog[i] = post[i];
    p.chain.n_instr = n_instr;
    for (int i = 0; i < n_instr; i++) p.chain.prog[i] = prog[i];
    p.n_ins = n_ins;
    p.R = R;
    p.out = (char*)out->data;
    p.out_dtype = out->dtype;
    p.square = (op == TADMA_REDUCE_SUMSQ || op == TADMA_REDUCE_RMS) ? 1 : 0;
    p.post = op == TADMA_REDUCE_MEAN ? POST_MEAN : op == TADMA_REDUCE_RMS ? POST_RMS : POST_NONE;
    const int kind = op == TADMA_REDUCE_MAX ? K_MAX : op == TADMA_REDUCE_MIN ? K_MIN
                   : op == TADMA_REDUCE_ARGMAX ? K_ARGMAX : op == TADMA_REDUCE_ARGMIN ? K_ARGMIN : K_SUM;
    // Kept dims, folded jointly for the operands and out.
    int64_t kd[TADMA_MAX_RANK], ks[1 + TADMA_MAX_INPUTS][TADMA_MAX_RANK];
    int kr = 0;
    for (int d = 0; d < rank; d++) {
        if (d == ax) continue;
        kd[kr] = S[d];
        ks[0][kr] = out->strides[keep ? d : (d < ax ? d : d - 1)];
        for (int k = 0; k < n_ins; k++) ks[1 + k][kr] = ins[k].dims[d] == 1 ? 0 : ins[k].strides[d];
        kr++;
    }
    int64_t nrows = 1;
    Folded f{};
    if (kr > 0) {
        f = fold(kr, kd, ks, 1 + n_ins);
        for (int d = 0; d < f.rank; d++) nrows *= f.dims[d];
    }
    p.nrows = nrows;
    p.krank = kr > 0 ? f.rank : 0;
    for (int d = 0; d < p.krank; d++) {
        p.kdm[d] = DivMod((uint64_t)f.dims[d]);
        p.kout[d] = f.strides[0][d];
        for (int k = 0; k < n_ins; k++) p.kin[k][d] = f.strides[1 + k][d];
    }
    bool vec = cm == TADMA_COMPUTE_F32 && R >= V;
    for (int k = 0; k < n_ins; k++) {
        Operand& o = p.chain.in[k];
        o.base = (const char*)ins[k].data;
        o.dtype = ins[k].dtype;
        o.streaming = 0;
        p.ax[k] = ins[k].dims[ax] == 1 ? 0 : ins[k].strides[ax];
        o.inner_bcast = p.ax[k] == 0 ? 1 : 0;
        if (p.ax[k] == 0) continue;
        const int es = dtype_size(o.dtype);
        const bool vdt = o.dtype == TADMA_F32 || o.dtype == TADMA_F16 || o.dtype == TADMA_BF16;
        bool ok = vdt && p.ax[k] == 1 && (uintptr_t)o.base % 16 == 0;
        for (int d = 0; d < p.krank && ok; d++) ok = (p.kin[k][d] * es) % 16 == 0;
        vec = vec && ok;
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (vec) {
        // Typed vector path when every streamed operand has one dtype.
        int sdt = -1;
        bool one_dt = true;
        for (int k = 0; k < n_ins; k++) {
            if (p.ax[k] == 0) continue;
            if (sdt < 0) sdt = ins[k].dtype;
            else if (ins[k].dtype != sdt) one_dt = false;
        }
        if (one_dt && sdt >= 0 && R >= 16 / dtype_size(sdt) && decode_fprog(prog, n_instr, n_ins, p.chain.fp))
            return launch_chain_reduce_typed(kind, sdt, p, s);
    }
    switch (cm) {
    case TADMA_COMPUTE_F32:
        return launch_chain_reduce_f32(kind, vec, p, s);
    case TADMA_COMPUTE_F64: return launch_chain_reduce_f64(kind, p, s);
    default: return launch_chain_reduce_i64(kind, p, s);
    }
}

extern "C" int tadma_b200_reduce_chain(int32_t op, const tadma_tensor* ins, int32_t n_ins, const tadma_instr* prog,
                                       int32_t n_instr, int32_t compute, int32_t axis, const tadma_tensor* out,
                                       void* stream) {
    return reduce_chain_impl(op, ins, n_ins, prog, n_instr, nullptr, 0, compute, axis, out, stream);
}

extern "C" int tadma_b200_reduce_chain_post(int32_t op, const tadma_tensor* ins, int32_t n_ins,
                                            const tadma_instr* prog, int32_t n_instr, const tadma_instr* post,
                                            int32_t n_post, int32_t compute, int32_t axis, const tadma_tensor* out,
                                            void* stream) {
    return reduce_chain_impl(op, ins, n_ins, prog, n_instr, post, n_post, compute, axis, out, stream);
}
