// fprog.cuh - pre-decoded fp32 chain programs for the typed chain kernels.
//
// A tadma_instr program is decoded once on the host into FInstr steps with
// one dense code each: the op, whether its second argument is the immediate
// or an operand, and every non-trivial rounding as a step of its own.  The
// device loop then reads 8 bytes per step and takes one jump-table branch,
// instead of testing the op class, the operand selector and the rounding
// type per instruction, and it runs each step on W elements at once (16 in
// the one- and two-operand kernels).  The op bodies are the ones the
// interpreter uses (ops.cuh), with the op a compile-time constant, so both
// paths give identical bits for the same chain.
#pragma once

#include <cstdint>

#include "kdiv.cuh"
#include "ops.cuh"

namespace tadma_b200 {

// Dense step codes.
constexpr int FC_FILL = 0;   // acc = imm (COPY of the immediate)
                             // 1..20: the unary op of the same number
constexpr int FC_BI = 21;    // FC_BI + (op - 32): binary op, imm second argument
constexpr int FC_BV = 41;    // FC_BV + (op - 32): binary op, operand `b` second argument
constexpr int FC_WHERE = 61; // acc = acc != 0 ? b : c (operands, or the imm where b / c < 0)
constexpr int FC_RND = 62;   // FC_RND + k: round to the k-th of F16, BF16, I64, I32, U8, BOOL, I8
constexpr int FC_SQR = 69;   // pow(acc, 2) with the immediate 2: one rounded multiply, as binary(POW) gives it
constexpr int FC_DIVK = 70;  // acc / imm through imm's reciprocal (kdiv.cuh), which the next step's imm holds
constexpr int FC_COUNT = 71;

struct FInstr {
    uint8_t code;
    int8_t b;  // operand of the second argument (FC_BV, FC_WHERE; < 0: the immediate)
    int8_t c;  // operand of WHERE's third argument (< 0: the immediate)
    uint8_t pad;
    float imm;  // the immediate rounded to fp32, as imm_as<float> rounds it
};

struct FProg {
    int32_t n;
    int32_t acc;  // the operand the accumulator starts from (ins[0] before any reordering)
    FInstr ins[2 * TADMA_MAX_INSTR];
};

// Host: decodes an fp32-compute program over `nin` operands.  `slot_of`
// (optional) renumbers the operands: ins[k] of the program is operand
// slot_of[k] of the kernel.  False when a step has no code (the caller keeps
// the run-time interpreter).
inline bool decode_fprog(const tadma_instr* prog, int n_instr, int nin, FProg& fp, const int* slot_of = nullptr) {
    static const int kRound[] = {TADMA_F16, TADMA_BF16, TADMA_I64, TADMA_I32, TADMA_U8, TADMA_BOOL, TADMA_I8};
    fp = FProg{};
    fp.acc = slot_of ? slot_of[0] : 0;
    auto emit = [&](int code, int b, int c, double imm) {
        FInstr& f = fp.ins[fp.n++];
        f.code = (uint8_t)code;
        f.b = (int8_t)b;
        f.c = (int8_t)c;
        f.imm = (float)imm;
    };
    auto slot = [&](int sel) { return sel >= 0 && sel < nin ? (slot_of ? slot_of[sel] : sel) : -1; };
    for (int i = 0; i < n_instr; i++) {
        const tadma_instr& I = prog[i];
        if (I.op >= 0 && I.op < 32) {
            if (I.op == TADMA_OP_COPY) {
                if (I.b == TADMA_SRC_IMM) emit(FC_FILL, -1, -1, I.imm);
            } else if (I.op <= TADMA_OP_NOT) {
                emit(I.op, -1, -1, 0.0);
            } else {
                return false;
            }
        } else if (I.op >= TADMA_OP_ADD && I.op <= TADMA_OP_LOR) {
            const int s = slot(I.b);
            // a division by an immediate inside kdiv's range takes a second
            // step for the reciprocal, while the remaining instructions
            // still fit at two steps each
            const bool kdiv = I.op == TADMA_OP_DIV && s < 0 && kdiv_in_range((float)I.imm) &&
                              2 * TADMA_MAX_INSTR - fp.n - 2 * (n_instr - i) >= 1;
            if (I.op == TADMA_OP_POW && s < 0 && (float)I.imm == 2.0f) {
                emit(FC_SQR, -1, -1, 0.0);
            } else if (kdiv) {
                const float b = (float)I.imm;
                emit(FC_DIVK, -1, -1, b);
                emit(FC_DIVK, -1, -1, 1.0f / b);  // RN(1/b): the host's IEEE single division
            } else {
                emit(s >= 0 ? FC_BV + (I.op - TADMA_OP_ADD) : FC_BI + (I.op - TADMA_OP_ADD), s, -1, I.imm);
            }
        } else if (I.op == TADMA_OP_WHERE) {
            emit(FC_WHERE, slot(I.b), slot(I.c), I.imm);
        } else {
            return false;
        }
        const int rd = I.round_dtype;
        if (rd >= 0 && rd != TADMA_F32 && rd != TADMA_F64) {
            int k = 0;
            while (k < 7 && kRound[k] != rd) k++;
            if (k == 7) return false;
            emit(FC_RND + k, -1, -1, 0.0);
        }
    }
    return true;
}

namespace {

// The unary op OP on one value: the interpreter's body (unary<FAST>) with
// the op fixed at compile time.  erf and log, common in ONNX graphs (GELU,
// log-softmax), are inlined; the rest of the out-of-line functions stay out
// of line.
template <int OP, bool FAST>
__device__ __forceinline__ float funary(float a) {
    if constexpr (OP == TADMA_OP_ERF) return erff(a);
    else if constexpr (OP == TADMA_OP_LOG) return logf(a);
    else return unary<FAST>(OP, a);
}

// An operand of a step: vector operands 0 .. NV-1 hold W values, scalar
// operands NV .. NV+NS-1 one value for all W (an innermost broadcast);
// sel < 0 is the step's immediate.
template <int NV, int NS, int W>
__device__ __forceinline__ void pick_or_imm(int sel, float imm, const float (&vv)[NV][W], const float (&sv)[NS > 0 ? NS : 1],
                                            float (&dst)[W]) {
    float s = imm;
#pragma unroll
    for (int k = 0; k < NS; k++)
        if (sel == NV + k) s = sv[k];
    bool vec = false;
#pragma unroll
    for (int k = 0; k < NV; k++) {
        if (sel == k) {
            vec = true;
#pragma unroll
            for (int j = 0; j < W; j++) dst[j] = vv[k][j];
        }
    }
    if (!vec) {
#pragma unroll
        for (int j = 0; j < W; j++) dst[j] = s;
    }
}

// Value j of operand sel (WHERE's third argument, chosen per element).
template <int NV, int NS, int W>
__device__ __forceinline__ float operand_at(int sel, float imm, const float (&vv)[NV][W], const float (&sv)[NS > 0 ? NS : 1],
                                            int j) {
    float v = imm;
#pragma unroll
    for (int k = 0; k < NV; k++)
        if (sel == k) v = vv[k][j];
#pragma unroll
    for (int k = 0; k < NS; k++)
        if (sel == NV + k) v = sv[k];
    return v;
}

#define TADMA_FU(OP)                                                        \
    case OP: {                                                              \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = funary<OP, FAST>(acc[j]); \
    } break;
#define TADMA_FB(OP)                                                        \
    case FC_BI + (OP - TADMA_OP_ADD): {                                     \
        const float s = I.imm;                                              \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = binary(OP, acc[j], s, s); \
    } break;                                                                \
    case FC_BV + (OP - TADMA_OP_ADD): {                                     \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = binary(OP, acc[j], bsel[j], bsel[j]); \
    } break;
#define TADMA_FR(K, DT)                                                     \
    case FC_RND + K: {                                                      \
        _Pragma("unroll") for (int j = 0; j < W; j++) acc[j] = round_to(acc[j], DT); \
    } break;

// Runs the decoded program on W values: the accumulator starts from operand
// fp.acc; NV vector operands, NS scalar ones.
template <int NV, int NS, int W, bool FAST>
__device__ __forceinline__ void run_fprog(const FProg& fp, float (&acc)[W], const float (&vv)[NV][W],
                                          const float (&sv)[NS > 0 ? NS : 1]) {
    pick_or_imm<NV, NS, W>(fp.acc, 0.0f, vv, sv, acc);
    for (int i = 0; i < fp.n; i++) {
        const FInstr I = fp.ins[i];
        // The second argument of a binary or WHERE step, picked once here
        // rather than in each case: one W-wide temporary for the whole switch.
        float bsel[W];
        if (I.code >= FC_BV && I.code <= FC_WHERE) pick_or_imm<NV, NS, W>(I.b, I.imm, vv, sv, bsel);
        switch (I.code) {
        case FC_FILL: {
#pragma unroll
            for (int j = 0; j < W; j++) acc[j] = I.imm;
        } break;
            TADMA_FU(TADMA_OP_NEG)
            TADMA_FU(TADMA_OP_ABS)
            TADMA_FU(TADMA_OP_EXP)
            TADMA_FU(TADMA_OP_LOG)
            TADMA_FU(TADMA_OP_SQRT)
            TADMA_FU(TADMA_OP_SIN)
            TADMA_FU(TADMA_OP_COS)
            TADMA_FU(TADMA_OP_TAN)
            TADMA_FU(TADMA_OP_ASIN)
            TADMA_FU(TADMA_OP_ACOS)
            TADMA_FU(TADMA_OP_ATAN)
            TADMA_FU(TADMA_OP_ASINH)
            TADMA_FU(TADMA_OP_ACOSH)
            TADMA_FU(TADMA_OP_ATANH)
            TADMA_FU(TADMA_OP_ERF)
            TADMA_FU(TADMA_OP_RELU)
            TADMA_FU(TADMA_OP_SIGMOID)
            TADMA_FU(TADMA_OP_TANH)
            TADMA_FU(TADMA_OP_GELU)
            TADMA_FU(TADMA_OP_NOT)
            TADMA_FB(TADMA_OP_ADD)
            TADMA_FB(TADMA_OP_SUB)
            TADMA_FB(TADMA_OP_MUL)
            TADMA_FB(TADMA_OP_DIV)
            TADMA_FB(TADMA_OP_POW)
            TADMA_FB(TADMA_OP_RSUB)
            TADMA_FB(TADMA_OP_RDIV)
            TADMA_FB(TADMA_OP_MAX)
            TADMA_FB(TADMA_OP_MIN)
            TADMA_FB(TADMA_OP_EQ)
            TADMA_FB(TADMA_OP_NE)
            TADMA_FB(TADMA_OP_LT)
            TADMA_FB(TADMA_OP_GT)
            TADMA_FB(TADMA_OP_LE)
            TADMA_FB(TADMA_OP_GE)
            TADMA_FB(TADMA_OP_AND)
            TADMA_FB(TADMA_OP_OR)
            TADMA_FB(TADMA_OP_XOR)
            TADMA_FB(TADMA_OP_LAND)
            TADMA_FB(TADMA_OP_LOR)
        case FC_WHERE: {
            // c is chosen per element, so no second W-wide temporary is live
#pragma unroll
            for (int j = 0; j < W; j++) acc[j] = acc[j] != 0.0f ? bsel[j] : operand_at<NV, NS, W>(I.c, I.imm, vv, sv, j);
        } break;
        case FC_SQR: {
#pragma unroll
            for (int j = 0; j < W; j++) acc[j] = __fmul_rn(acc[j], acc[j]);
        } break;
        case FC_DIVK: {
            const KnownDivisor kd{I.imm, fp.ins[i + 1].imm, true};
            i++;  // the reciprocal's step
            bool fast = true;
#pragma unroll
            for (int j = 0; j < W; j++) fast = fast & kdiv_in_range(acc[j]);
            if (fast) {
#pragma unroll
                for (int j = 0; j < W; j++) acc[j] = kdiv_fast(acc[j], kd);
            } else {
#pragma unroll
                for (int j = 0; j < W; j++) acc[j] = __fdiv_rn(acc[j], kd.b);
            }
        } break;
            TADMA_FR(0, TADMA_F16)
            TADMA_FR(1, TADMA_BF16)
            TADMA_FR(2, TADMA_I64)
            TADMA_FR(3, TADMA_I32)
            TADMA_FR(4, TADMA_U8)
            TADMA_FR(5, TADMA_BOOL)
            TADMA_FR(6, TADMA_I8)
        default:
            break;
        }
    }
}

#undef TADMA_FU
#undef TADMA_FB
#undef TADMA_FR

// The same on NIN vector operands.
template <int NIN, int W, bool FAST>
__device__ __forceinline__ void run_fprog(const FProg& fp, float (&acc)[W], const float (&val)[NIN][W]) {
    const float none[1] = {0.0f};
    run_fprog<NIN, 0, W, FAST>(fp, acc, val, none);
}

}  // namespace
}  // namespace tadma_b200
