/*
 * tadma_b200.h - C ABI of the B200 (sm_100a) kernels behind TADMA's Tensor API.
 *
 * Plain pointers, sizes and PODs only; no C++ or torch types. Every entry point
 * is asynchronous on the `stream` argument (a cudaStream_t passed as void*,
 * NULL = legacy default stream), exactly as every TADMA op is asynchronous on
 * the thread-local `tadma::stream` (reference include/tadma/Globals.hpp:8).
 *
 * Return value: TADMA_OK or a TADMA_ERR_* code.  Host-side validation errors
 * (bad rank, mismatched dims, unsupported dtype) are returned synchronously and
 * launch nothing; tadma_b200_last_error() gives the message of the calling
 * thread's last failure.  This is the C counterpart of the reference's
 * check_cuda()/std::runtime_error convention (include/tadma/Defines.hpp:14-26).
 *
 * Device-side data errors (a gather id outside [-n, n)) cannot be returned by
 * an async call: the kernel sets a bit in a per-device error word and writes
 * zeros for that row; tadma_b200_error_flags() reads (and optionally clears)
 * that word after synchronising.
 *
 * Every kernel is launched with programmatic stream serialisation: it may be
 * scheduled while the previous kernel of its stream drains, and it waits for
 * that kernel to complete before touching memory, so stream order is kept.
 * Calls may be captured into a CUDA graph (prepare them on the capture
 * stream); tadma_b200_reduce's split path allocates a stream-ordered
 * workspace (cudaMallocAsync), tadma_b200_reduce_noalloc does not.
 */
#ifndef TADMA_B200_H
#define TADMA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- dtypes -- */
/* Element types. The reference takes T from C++ (float, __half, int64_t, bool,
 * uint8_t ... : Operations.hpp:67-89); bf16 is new (it has no bf16). */
enum tadma_dtype {
    TADMA_F32 = 0,
    TADMA_F16 = 1,
    TADMA_BF16 = 2,
    TADMA_F64 = 3,
    TADMA_I64 = 4,
    TADMA_I32 = 5,
    TADMA_U8 = 6,
    TADMA_BOOL = 7, /* 1 byte, 0 or 1 */
    TADMA_I8 = 8
};

enum tadma_status {
    TADMA_OK = 0,
    TADMA_ERR_INVALID = 1,     /* bad argument: rank, dims, null pointer, dtype mix */
    TADMA_ERR_UNSUPPORTED = 2, /* valid but not implemented (e.g. exp on int64 compute) */
    TADMA_ERR_CUDA = 3,        /* a CUDA runtime call failed */
    TADMA_ERR_INDEX = 4        /* device error word: gather id out of range */
};

#define TADMA_MAX_RANK 8

/* A strided view, the runtime image of Tensor<T, Allocator, Sequence<dims...>,
 * Sequence<strides...>> (reference Tensor.hpp:20-40).  Strides are in
 * elements; stride 0 marks a broadcast dimension (Tensor.hpp:323-336).
 * `data` points at element (0,...,0).  rank 0 = scalar (one element). */
typedef struct tadma_tensor {
    void* data;
    int32_t dtype;
    int32_t rank;
    int64_t dims[TADMA_MAX_RANK];
    int64_t strides[TADMA_MAX_RANK];
} tadma_tensor;

/* ------------------------------------------------------- element-wise ops -- */
/* Op codes of one chain instruction.  Unary codes map acc -> f(acc); binary
 * codes map acc -> f(acc, b); WHERE maps acc -> acc ? b : c.  The set is the
 * reference's MKOP list (Operations.hpp:166-182), pow (:186-188), the tensor /
 * scalar operators (Tensor.hpp:494-540) and where (Operations.hpp:235-242). */
enum tadma_op {
    /* unary */
    TADMA_OP_COPY = 0, /* identity: a cast when in/out dtypes differ (to<U>, contiguous) */
    TADMA_OP_NEG = 1,
    TADMA_OP_ABS = 2,
    TADMA_OP_EXP = 3,
    TADMA_OP_LOG = 4,
    TADMA_OP_SQRT = 5,
    TADMA_OP_SIN = 6,
    TADMA_OP_COS = 7,
    TADMA_OP_TAN = 8,
    TADMA_OP_ASIN = 9,
    TADMA_OP_ACOS = 10,
    TADMA_OP_ATAN = 11,
    TADMA_OP_ASINH = 12,
    TADMA_OP_ACOSH = 13,
    TADMA_OP_ATANH = 14,
    TADMA_OP_ERF = 15,
    TADMA_OP_RELU = 16,
    TADMA_OP_SIGMOID = 17,
    TADMA_OP_TANH = 18,
    TADMA_OP_GELU = 19, /* tanh form, constants of Operations.hpp:181 */
    TADMA_OP_NOT = 20,  /* logical not: acc == 0 */
    /* binary: acc = acc (op) b */
    TADMA_OP_ADD = 32,
    TADMA_OP_SUB = 33,
    TADMA_OP_MUL = 34,
    TADMA_OP_DIV = 35,
    TADMA_OP_POW = 36,
    TADMA_OP_RSUB = 37, /* b - acc  (scalar - tensor, Tensor.hpp:504) */
    TADMA_OP_RDIV = 38, /* b / acc  (scalar / tensor, Tensor.hpp:505) */
    TADMA_OP_MAX = 39,
    TADMA_OP_MIN = 40,
    TADMA_OP_EQ = 41,
    TADMA_OP_NE = 42,
    TADMA_OP_LT = 43,
    TADMA_OP_GT = 44,
    TADMA_OP_LE = 45,
    TADMA_OP_GE = 46,
    TADMA_OP_AND = 47, /* bitwise (integer compute) / logical (float compute) */
    TADMA_OP_OR = 48,
    TADMA_OP_XOR = 49,
    TADMA_OP_LAND = 50,
    TADMA_OP_LOR = 51,
    /* ternary */
    TADMA_OP_WHERE = 64 /* acc = (acc != 0) ? b : c */
};

/* Operand selector: >= 0 selects ins[k]; TADMA_SRC_IMM selects instr.imm. */
#define TADMA_SRC_IMM (-1)
#define TADMA_SRC_NONE (-2)

/* One instruction of a fused element-wise chain.  After the op, when
 * `round_dtype` >= 0 the accumulator is rounded to that dtype: this reproduces
 * the reference's materialised intermediate (every node writes a tensor of
 * dtype decltype(f(T)), Kernels.hpp:20-45) inside one fused kernel. */
typedef struct tadma_instr {
    int32_t op;
    int32_t b; /* operand selector of the 2nd argument (binary / WHERE) */
    int32_t c; /* operand selector of the 3rd argument (WHERE) */
    int32_t round_dtype;
    double imm;
} tadma_instr;

/* Compute (accumulator) type of a chain. */
enum tadma_compute {
    TADMA_COMPUTE_AUTO = -1, /* F64 if any operand is f64/i64 and no float op needs F32, else F32 */
    TADMA_COMPUTE_F32 = 0,
    TADMA_COMPUTE_F64 = 1,
    TADMA_COMPUTE_I64 = 2,
    /* fp32 without the fast-math bodies: an fp32 chain with a 16-bit output
     * otherwise evaluates exp / sigmoid / gelu with the SFU exponential and
     * reciprocal (error far below half a 16-bit ulp); this mode keeps the
     * precise bodies, as a chain whose transcendental steps each round to fp32
     * needs to equal those steps made as separate calls */
    TADMA_COMPUTE_F32_PRECISE = 3
};

#define TADMA_MAX_INPUTS 6
#define TADMA_MAX_INSTR 16

/*
 * Fused element-wise chain: out[i] = chain(ins[0][i], ins[1][i], ...).
 * acc starts as ins[0] converted to the compute type; each instruction updates
 * acc; out = acc converted to out->dtype.  All tensors have out's rank and dims
 * (broadcast operands carry stride 0), so `out` fixes the execution shape as
 * t0::Dims does in CombineVariadicNode (Kernels.hpp:10-14).  out may alias
 * ins[0] with equal strides (the in-place form, Kernels.hpp:16-18).
 * n_ins = 0 is allowed when the chain starts from instr[0].imm via COPY with
 * b = TADMA_SRC_IMM (a fill, Tensor.hpp:284-286).
 *
 * Replaces: EltwiseNode / CombineToNode / CombineNode / InplaceNode /
 * MakeEltwiseNode (Kernels.hpp:16-53), the executor CUDAHIPExecutor +
 * CUDAHIPExecutorKernel (Node.hpp:25-48) and, for linear chains, MergeNodes
 * (Node.hpp:189-224).
 */
int tadma_b200_eltwise(const tadma_tensor* out, const tadma_tensor* ins, int32_t n_ins,
                       const tadma_instr* prog, int32_t n_instr, int32_t compute, void* stream);

/* ------------------------------------------------------------- reductions -- */
enum tadma_reduce_op {
    TADMA_REDUCE_SUM = 0,
    TADMA_REDUCE_MEAN = 1, /* sum / n  (Tensor.hpp:448, post = x / Dim(D)) */
    TADMA_REDUCE_MAX = 2,
    TADMA_REDUCE_MIN = 3,
    TADMA_REDUCE_ARGMAX = 4, /* int64 index, first occurrence; NaN counts as max */
    TADMA_REDUCE_ARGMIN = 5, /* int64 index, first occurrence; NaN counts as min */
    TADMA_REDUCE_SUMSQ = 6,  /* sum of squares (rms_norm's pre-op, Operations.hpp:223-226) */
    TADMA_REDUCE_RMS = 7     /* sqrt(mean(x^2)) (rms_norm's reduction, Operations.hpp:223-226) */
};

/*
 * Reduce `in` along `axis` (negative counts from the end) into `out`.
 * out has either in's rank with dims[axis] = 1 (KeepDims = true, the
 * reference default) or rank-1 with that dim removed (KeepDims = false).
 * `pre_op` is a unary tadma_op applied to each element before reducing
 * (TADMA_OP_COPY for none), e.g. EXP for sum(exp(x)).  Float inputs accumulate
 * in fp32 (fp64 for f64 input), integer inputs in int64.
 *
 * Replaces: ReduceNode + ReduceKernel (kernels/Reduce.hpp:10-71) behind
 * Tensor::reduce / sum / min / max / mean (Tensor.hpp:436-448); ARGMAX/ARGMIN
 * are new (the reference has none).
 */
int tadma_b200_reduce(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op,
                      const tadma_tensor* out, void* stream);

/*
 * Reduction of a fused element-wise chain, in one kernel:
 *   out = reduce_op over `axis` of chain(ins[0][i], ins[1][i], ...)
 * The chain (prog, n_instr, compute: as tadma_b200_eltwise) is evaluated per
 * element on the way into the reduction and never materialised.  All ins have
 * the same rank and dims S (broadcast operands carry stride 0); out has S
 * with dims[axis] = 1 (KeepDims) or that dim removed.  op and the out dtype
 * follow tadma_b200_reduce; float chains reduce in the compute type (fp32 for
 * TADMA_COMPUTE_F32, fp64 for F64), integer chains in int64.  The result
 * equals tadma_b200_eltwise into a compute-type temporary followed by
 * tadma_b200_reduce (bit for bit for max / min / argmax / argmin; sums within
 * the fp32 reduction tolerance, their order differing).
 *
 * Replaces: an EltwiseNode / CombineToNode chain feeding a ReduceNode
 * (Kernels.hpp:20-45 -> kernels/Reduce.hpp:10-71), i.e. the ReduceKernel
 * pre-functor (Reduce.hpp:29-56) generalised from one unary op to a chain
 * over up to 6 broadcast operands; e.g. sum<-1>(exp(A + b)) in one launch.
 */
int tadma_b200_reduce_chain(int32_t op, const tadma_tensor* ins, int32_t n_ins, const tadma_instr* prog,
                            int32_t n_instr, int32_t compute, int32_t axis, const tadma_tensor* out,
                            void* stream);

/*
 * tadma_b200_reduce_chain followed by a chain on each reduced value:
 * out = post(reduce(chain(ins...))).  `post` holds up to TADMA_MAX_INSTR
 * instructions whose operands are immediates (b / c = TADMA_SRC_IMM or
 * TADMA_SRC_NONE); it runs in the compute type on the value the reduction
 * would store (after MEAN's division / RMS's square root), each instruction
 * rounding to its round_dtype, then the result is stored to out->dtype.  Not
 * for ARGMAX / ARGMIN.  One kernel: a variance and the + eps and sqrt that
 * make it a layer_norm denominator never round-trip through HBM.
 * Replaces: ReduceKernel's post functor (kernels/Reduce.hpp:29-56, the sqrt
 * post of layer_norm's standard deviation, Operations.hpp:195-203),
 * generalised to a chain, plus the eager nodes that follow a reduction.
 */
int tadma_b200_reduce_chain_post(int32_t op, const tadma_tensor* ins, int32_t n_ins, const tadma_instr* prog,
                                 int32_t n_instr, const tadma_instr* post, int32_t n_post, int32_t compute,
                                 int32_t axis, const tadma_tensor* out, void* stream);

/*
 * One pass over the rows of a [rows, cols] grid: per-row reductions of
 * element chains (stages), then an element-wise chain that may read them.
 * A LayerNorm, RMSNorm or softmax written as separate ops (mean, -, pow,
 * mean, + eps, sqrt, /, *, + as generated code spells it) runs as one
 * kernel that reads each row once, with the bits of the separate calls.
 *
 * Operands (prog / stage chains select them by number):
 *   0 .. n_ins - 1        ins[k], each a rank-2 view of the grid: dims
 *                         {rows or 1, cols or 1}, strides {rs, cs}:
 *                         a row operand (cs = 1, rs != 0), a column operand
 *                         (rows dim 1 or rs = 0, cs = 1) or a row scalar
 *                         (cols dim 1 or cs = 0);
 *   n_ins + s             the value stage s stored for the row (after its
 *                         post chain and the rounding to its out dtype),
 *                         readable by later stages and by prog.
 * Each stage is tadma_b200_reduce_chain_post over the last axis with op
 * SUM, MEAN, MAX or MIN, fp32 compute; its out holds rows values (a rank-1
 * view {rows} with its stride).  prog runs in fp32 (TADMA_COMPUTE_F32, or
 * TADMA_COMPUTE_F32_PRECISE: as tadma_b200_eltwise) and writes out, a
 * {rows, cols} view with unit column stride.
 *
 * Limits: cols a multiple of 16 / dtype size, at most 32 x 8 x that (1024
 * fp32, 2048 fp16 / bf16 values); at most 2 row operands and 2 column
 * operands, all of one float dtype, 16-byte aligned rows; at most 2 row
 * scalars (any float dtype); at most TADMA_ROWPROG_MAX_STAGES stages; out
 * F32, F16 or BF16.  Other grids return TADMA_ERR_UNSUPPORTED with nothing
 * launched: the caller runs the ops one by one.
 *
 * The result equals the separate calls bit for bit: each stage folds in the
 * order of the row reductions (lane l of a warp takes 16-byte vectors l,
 * l + 32, ... in order, then the fixed lane butterfly), the chains use the
 * element-wise engine's op bodies and roundings.
 * Replaces: the ReduceNode / EltwiseNode sequence of a decomposed
 * normalisation (Kernels.hpp:20-45, kernels/Reduce.hpp:10-71), as
 * layer_norm / softmax compose it (Operations.hpp:190-220).
 */
#define TADMA_ROWPROG_MAX_STAGES 3
typedef struct tadma_row_stage {
    int32_t op; /* TADMA_REDUCE_SUM, MEAN, MAX or MIN */
    int32_t n_instr;
    int32_t n_post;
    int32_t acc;                       /* the operand the element chain starts from */
    tadma_instr prog[TADMA_MAX_INSTR]; /* element chain */
    tadma_instr post[TADMA_MAX_INSTR]; /* on the reduced value, immediates only */
    tadma_tensor out;                  /* rank 1, rows values */
} tadma_row_stage;

typedef struct tadma_row_program {
    int64_t rows, cols;
    int32_t n_ins;
    int32_t n_stages;
    int32_t n_instr;
    int32_t compute; /* TADMA_COMPUTE_F32 or TADMA_COMPUTE_F32_PRECISE */
    int32_t acc;     /* the operand the final chain starts from */
    int32_t pad;
    tadma_tensor ins[TADMA_MAX_INPUTS];
    tadma_row_stage stages[TADMA_ROWPROG_MAX_STAGES];
    tadma_instr prog[TADMA_MAX_INSTR]; /* the final chain */
    tadma_tensor out;                  /* rank 2 {rows, cols} */
} tadma_row_program;

int tadma_b200_row_program(const tadma_row_program* rp, void* stream);

/*
 * tadma_b200_reduce without any device allocation.  No counterpart in the
 * reference.  For callers that cannot call cudaMalloc: a process whose memory
 * pool has already claimed the device's HBM (so any further allocation
 * fails), a latency-critical path that must not enter the allocator, or a
 * host that only lends the library the buffers it passes in.
 * Same arguments and errors as tadma_b200_reduce, results within the same
 * tolerance.  Reductions that split a long axis across CTAs keep their
 * partial results in a 2 MiB static device buffer inside the library (every
 * GPU that loads the library holds it until the process exits) instead of a
 * per-call workspace.  When the split that tadma_b200_reduce would choose
 * needs more than 2 MiB of partials, this entry point splits the axis into
 * fewer parts, so that they fit, or reduces it in one pass (no partials);
 * every shape therefore runs, possibly slower than tadma_b200_reduce, and
 * summed in a different order (a different rounding of the same sum).
 * - The first call on a device looks up the buffer's device address
 *   (cudaGetSymbolAddress) and caches it; make that first call outside any
 *   stream capture.
 * - Every call shares the one buffer and overwrites what the previous call
 *   left there (nothing in it needs to start at zero); calls whose executions
 *   overlap on the GPU (different streams, no ordering) race on it.
 */
int tadma_b200_reduce_noalloc(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op,
                              const tadma_tensor* out, void* stream);

/* ---------------------------------------------- fused reduce + broadcast -- */
/*
 * Softmax along `axis`: out = exp(x - max) / sum(exp(x - max)), one read and
 * one write of the data, fp32 math.  Mathematically equal to the reference's
 * exp -> sum -> divide composition, which has no max subtraction
 * (Operations.hpp:190-193).  out may alias in (the Inplace = true form).
 */
int tadma_b200_softmax(const tadma_tensor* in, int32_t axis, const tadma_tensor* out, void* stream);

enum tadma_norm_mode {
    TADMA_LN_ONNX = 0, /* (x - mean) / sqrt(var + eps) * gamma + beta (ONNX LayerNormalization) */
    TADMA_LN_TADMA = 1 /* (x - mean) / (sqrt(var) + eps) * gamma + beta (Operations.hpp:205-220) */
};

/*
 * LayerNorm over the last `axis` (must be the last dimension, contiguous).
 * gamma/beta are 1-D of that length (or data == NULL for 1 / 0).
 * var is the population variance.  out may alias in.
 * Replaces: mean_stddev + layer_norm (Operations.hpp:195-220).
 */
int tadma_b200_layer_norm(const tadma_tensor* in, int32_t axis, const tadma_tensor* gamma,
                          const tadma_tensor* beta, double eps, int32_t mode,
                          const tadma_tensor* out, void* stream);

/*
 * RMSNorm over the last axis: out = x / sqrt(mean(x^2) + eps) (eps = 0 is the
 * reference formula, Operations.hpp:222-233).  out may alias in.
 */
int tadma_b200_rms_norm(const tadma_tensor* in, int32_t axis, double eps, const tadma_tensor* out,
                        void* stream);

/* ----------------------------------------------------------------- gather -- */
/*
 * ONNX Gather along `axis` with an optional fused broadcast add:
 *   out[i_pre, j..., i_post] = table[i_pre, ids[j...], i_post] (+ add[...])
 * out dims = table.dims[:axis] ++ ids.dims ++ table.dims[axis+1:].
 * ids are int64 or int32; a negative id counts from the end (ONNX); an id
 * outside [-n, n) sets TADMA_ERR_INDEX in the device error word and yields
 * zeros (plus `add`) for that slice.  `add` (data == NULL for none) has out's
 * rank and dims with stride 0 on broadcast dims.  Math is fp32, rounded once
 * to out->dtype.
 * Replaces: gather (Operations.hpp:244-262) + EltwiseVariadicNDNode /
 * EltwiseVariadicNDKernel (kernels/EltwiseVariadicND.hpp:6-38), and fuses the
 * following CombineToNode add (Kernels.hpp:33-45).
 */
int tadma_b200_gather(const tadma_tensor* table, int32_t axis, const tadma_tensor* ids,
                      const tadma_tensor* add, const tadma_tensor* out, void* stream);

/* ------------------------------------------------------- seeded generator -- */
enum tadma_dist {
    TADMA_DIST_UNIFORM = 0, /* U(p0, p1) from a 24-bit grid: p0 + (p1 - p0) * k * 2^-24 */
    TADMA_DIST_NORMAL = 1,  /* N(p0, p1^2): Box-Muller in double from two 53-bit uniforms, |z| < 8.6 */
    TADMA_DIST_INDEX = 2    /* integers in [0, p1) (p0 ignored), int64/int32 out */
};

/*
 * Fill a contiguous tensor with the counter-based seeded generator: element i
 * (global index `offset + i`) is a pure function of (seed, stream_id, offset+i),
 * so any shard of a tensor is generated bit-identically on any GPU count and
 * by the host oracle.  No counterpart in the reference (its randn,
 * Operations.hpp:290-297, is host-only and unseeded).
 */
int tadma_b200_fill(const tadma_tensor* out, int32_t dist, double p0, double p1, uint64_t seed,
                    uint64_t stream_id, int64_t offset, void* stream);

/* --------------------------------------------------------------- runtime -- */
/* Message of the calling thread's last failed call ("" if none). */
const char* tadma_b200_last_error(void);
/* Library version string. */
const char* tadma_b200_version(void);
/* Synchronise the current device and read its device error word (bit
 * (1 << TADMA_ERR_INDEX) = bad gather id).  clear != 0 resets it.  Returns
 * TADMA_OK or TADMA_ERR_CUDA. */
int tadma_b200_error_flags(uint32_t* flags, int32_t clear);
/* Bytes per element of a dtype, 0 for an unknown code. */
int32_t tadma_b200_dtype_size(int32_t dtype);

#ifdef __cplusplus
}
#endif

#endif /* TADMA_B200_H */
