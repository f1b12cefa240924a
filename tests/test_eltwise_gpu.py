"""Fused element-wise chains (tadma_b200_eltwise) vs the oracle (or_eltwise).

Tolerances (north star: element-wise float output bit-exact where the op order
matches, otherwise within 1 ulp):
* +, -, *, /, comparisons, where, relu, neg, abs, sqrt, copy/cast, pow(x, 2):
  bit-exact (both sides round once per op, no contraction);
* transcendental ops computed in fp32 (COMPUTE_F32) with fp16/bf16 output:
  <= 1 ulp of the output type;
* transcendental ops with fp32 output: COMPUTE_F64 <= 1 ulp; COMPUTE_F32 is
  bounded by CUDA's fp32 math library (per-op table below, e.g. expf 2 ulp).
"""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, Op, instr, make_tensor
from tests.helpers import dev_view, empty_dev, from_dev, gen, to_dev, ulp_diff

pytestmark = pytest.mark.gpu

F32_ULP = {Op.EXP: 2, Op.LOG: 2, Op.SQRT: 0, Op.SIN: 2, Op.COS: 2, Op.TAN: 4, Op.ASIN: 4, Op.ACOS: 4,
           Op.ATAN: 4, Op.ASINH: 4, Op.ACOSH: 4, Op.ATANH: 4, Op.ERF: 4, Op.SIGMOID: 4, Op.TANH: 4,
           Op.GELU: 64}

DOMAIN = {Op.LOG: (0.01, 50.0), Op.SQRT: (0.0, 50.0), Op.ASIN: (-1.0, 1.0), Op.ACOS: (-1.0, 1.0),
          Op.ACOSH: (1.0, 30.0), Op.ATANH: (-0.99, 0.99), Op.TAN: (-1.5, 1.5)}


def run_both(out_shape, out_dt, ins, prog, compute=Compute.AUTO):
    """ins: list of (numpy array, dtype). Returns (device result, oracle result)."""
    views = [dev_view(a, dt) for a, dt in ins]
    out = empty_dev(out_shape, out_dt)
    tb.eltwise(out, [d for _, d in views], prog, compute)
    ref = np.zeros(out_shape, dtype=from_dev(out).dtype)
    rc = O.eltwise(ref, [a for a, _ in ins], prog, compute, out_dtype=out_dt, in_dtypes=[dt for _, dt in ins])
    assert rc == 0
    return from_dev(out), ref


def uniform(shape, lo, hi, dt=DType.F32, sid=1):
    return gen(shape, dt, Dist.UNIFORM, lo, hi, sid)


@pytest.mark.parametrize("op", [op for op in Op if op < 32 and op != Op.COPY])
@pytest.mark.parametrize("out_dt", [DType.F32, DType.BF16, DType.F16])
def test_unary_f32_compute(op, out_dt):
    lo, hi = DOMAIN.get(op, (-6.0, 6.0))
    x = uniform((129, 257), lo, hi)
    got, ref = run_both(x.shape, out_dt, [(x, DType.F32)], [instr(op)], Compute.F32)
    d = ulp_diff(got, ref, out_dt)
    if out_dt == DType.F32:
        tol = F32_ULP.get(op, 0)
    else:
        tol = 1 if op in F32_ULP else 0
    assert d.max() <= tol, f"{op.name} -> {out_dt.name}: max ulp {d.max()} (tol {tol})"


@pytest.mark.parametrize("op", sorted(F32_ULP, key=int))
def test_unary_f64_compute_f32_out_within_1ulp(op):
    lo, hi = DOMAIN.get(op, (-6.0, 6.0))
    x = uniform((64, 129), lo, hi)
    got, ref = run_both(x.shape, DType.F32, [(x, DType.F32)], [instr(op)], Compute.F64)
    d = ulp_diff(got, ref, DType.F32)
    assert d.max() <= 1, f"{op.name}: max ulp {d.max()}"


@pytest.mark.parametrize("op", [Op.ADD, Op.SUB, Op.MUL, Op.DIV, Op.RSUB, Op.RDIV, Op.MAX, Op.MIN, Op.EQ, Op.NE,
                                Op.LT, Op.GT, Op.LE, Op.GE, Op.AND, Op.OR, Op.XOR, Op.LAND, Op.LOR, Op.POW])
def test_binary_broadcast_bit_exact(op):
    # x[33, 1030] (op) y[1030] broadcast over rows, bf16 y, fp32 out.
    x = gen((33, 1030), DType.F32, Dist.NORMAL, 0.0, 2.0, 3)
    y = gen((1, 1030), DType.BF16, Dist.NORMAL, 0.0, 2.0, 4)
    if op == Op.POW:
        x = np.abs(x) + np.float32(0.5)
    y_view = np.broadcast_to(y, (33, 1030))
    prog = [instr(op, b=1)] if op != Op.POW else [instr(Op.POW, b=SRC_IMM, imm=2.0)]
    got, ref = run_both((33, 1030), DType.F32, [(x, DType.F32), (y_view, DType.BF16)], prog, Compute.F32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"{op.name}: {(got != ref).sum()} mismatches"


def test_config1_chain_add_exp():
    # Config 1 first stage: E = exp(A + b), A[64,128], b[128] ~ N(0,1), seed 0.
    A = gen((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 1)
    b = gen((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 2)
    bv = np.broadcast_to(b[None, :], (64, 128))
    prog = [instr(Op.ADD, b=1, round_dtype=DType.F32), instr(Op.EXP, round_dtype=DType.F32)]
    got, ref = run_both((64, 128), DType.F32, [(A, DType.F32), (bv, DType.F32)], prog, Compute.F32)
    assert ulp_diff(got, ref, DType.F32).max() <= 2
    got64, ref64 = run_both((64, 128), DType.F32, [(A, DType.F32), (bv, DType.F32)], prog, Compute.F64)
    assert ulp_diff(got64, ref64, DType.F32).max() <= 1


def config2_prog():
    # y = gelu(x * s + bias): float nodes x*s and +bias, gelu, bf16 store.
    return [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
            instr(Op.GELU, round_dtype=DType.F32)]


@pytest.mark.parametrize("rows,cols", [(64, 8192), (37, 1000), (3, 24)])
def test_config2_chain_small(rows, cols):
    x = gen((rows, cols), DType.BF16, Dist.NORMAL, 0.0, 1.0, 1)
    bias = gen((cols,), DType.BF16, Dist.NORMAL, 0.0, 0.1, 2)
    got, ref = run_both((rows, cols), DType.BF16, [(x, DType.BF16), (np.broadcast_to(bias, (rows, cols)), DType.BF16)],
                        config2_prog(), Compute.F32)
    d = ulp_diff(got, ref, DType.BF16)
    assert d.max() <= 1
    # the straightforward per-config loop agrees with the generic oracle chain bit for bit
    ref2 = np.zeros_like(ref)
    xb, bb = np.ascontiguousarray(x), np.ascontiguousarray(bias)
    O.lib().or_cfg2_gelu_affine_bf16(O.ptr(xb), O.ptr(bb), 0.5, O.ptr(ref2), rows, cols)
    assert np.array_equal(ref2, ref)


def test_config2_full_size():
    # BASELINE config 2 at full size: x[8192, 8192] bf16, bias[8192] bf16, s = 0.5.
    import torch
    rows = cols = 8192
    x = empty_dev((rows, cols), DType.BF16)
    bias = empty_dev((cols,), DType.BF16)
    tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=1)
    tb.fill(bias, Dist.NORMAL, 0.0, 0.1, seed=0, stream_id=2)
    y = empty_dev((rows, cols), DType.BF16)
    bview = make_tensor(bias.data_ptr(), DType.BF16, [rows, cols], [0, 1])
    tb.eltwise(y, [x, bview], config2_prog(), Compute.F32)
    torch.cuda.synchronize()
    xh, bh, got = from_dev(x), from_dev(bias), from_dev(y)
    ref = np.zeros_like(got)
    O.lib().or_cfg2_gelu_affine_bf16(O.ptr(xh), O.ptr(bh), 0.5, O.ptr(ref), rows, cols)
    d = ulp_diff(got, ref, DType.BF16)
    assert d.max() <= 1
    assert (d == 0).mean() > 0.999


def test_odd_sizes_and_tail():
    for n in (1, 7, 8, 9, 1000003):
        x = uniform((n,), -3, 3, sid=n)
        got, ref = run_both((n,), DType.F32, [(x, DType.F32)], [instr(Op.MUL, b=SRC_IMM, imm=3.0), instr(Op.RELU)],
                            Compute.F32)
        assert np.array_equal(got, ref), n


def test_strided_transposed_input():
    x = uniform((96, 80), -2, 2)
    xt = x.T  # non-contiguous view, strides (1, 80)
    got, ref = run_both((80, 96), DType.F32, [(np.ascontiguousarray(xt), DType.F32)], [instr(Op.NEG)], Compute.F32)
    # device: read through the transposed strides directly
    import torch
    xd = to_dev(x)
    out = empty_dev((80, 96), DType.F32)
    tb.eltwise(out, [make_tensor(xd.data_ptr(), DType.F32, [80, 96], [1, 80])], [instr(Op.NEG)], Compute.F32)
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(out), -xt)
    assert np.array_equal(got, ref)


def test_inplace():
    import torch
    x = uniform((1024, 64), -2, 2)
    xd = to_dev(x)
    tb.eltwise(xd, [xd], [instr(Op.MUL, b=SRC_IMM, imm=2.0), instr(Op.ADD, b=SRC_IMM, imm=1.0)], Compute.F32)
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(xd), (x * np.float32(2)) + np.float32(1))


def test_where_and_bool_out():
    c = gen((50, 64), DType.F32, Dist.UNIFORM, -1, 1, 5) > 0
    x = uniform((50, 64), -1, 1, sid=6)
    y = uniform((50, 64), -1, 1, sid=7)
    got, ref = run_both((50, 64), DType.F32, [(c, DType.BOOL), (x, DType.F32), (y, DType.F32)],
                        [instr(Op.WHERE, b=1, c=2)])
    assert np.array_equal(got, ref) and np.array_equal(got, np.where(c, x, y))
    got, ref = run_both((50, 64), DType.BOOL, [(x, DType.F32), (y, DType.F32)], [instr(Op.GT, b=1)])
    assert np.array_equal(got, ref) and np.array_equal(got, x > y)


def test_int64_compute():
    a = gen((10, 100), DType.I64, Dist.INDEX, 0, 1 << 40, 8) - (1 << 39)
    b = gen((10, 100), DType.I64, Dist.INDEX, 0, 1000, 9) - 500
    prog = [instr(Op.MUL, b=SRC_IMM, imm=3), instr(Op.DIV, b=1), instr(Op.NEG)]
    got, ref = run_both((10, 100), DType.I64, [(a, DType.I64), (b, DType.I64)], prog)
    assert np.array_equal(got, ref)


def test_f64_compute():
    x = gen((33, 65), DType.F64, Dist.NORMAL, 0, 1, 10)
    got, ref = run_both((33, 65), DType.F64, [(x, DType.F64)], [instr(Op.MUL, b=SRC_IMM, imm=1.5),
                                                               instr(Op.ADD, b=SRC_IMM, imm=-0.25)])
    assert np.array_equal(got, ref)


def test_fill_from_immediate():
    import torch
    out = empty_dev((17, 3), DType.F16)
    tb.eltwise(out, [], [instr(Op.COPY, b=SRC_IMM, imm=1.5)])
    torch.cuda.synchronize()
    assert np.all(from_dev(out) == np.float16(1.5))


def test_cast_chain_rounding():
    # round_dtype reproduces a materialised fp16 intermediate inside one kernel
    x = uniform((257,), -100, 100)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=1.0 / 3.0, round_dtype=DType.F16), instr(Op.MUL, b=SRC_IMM, imm=3.0)]
    got, ref = run_both((257,), DType.F32, [(x, DType.F32)], prog, Compute.F32)
    assert np.array_equal(got, ref)


def test_invalid_arguments_raise():
    out = empty_dev((4, 4), DType.F32)
    x = empty_dev((4, 5), DType.F32)
    with pytest.raises(tb.TadmaError):
        tb.eltwise(out, [x], [instr(Op.NEG)])
    with pytest.raises(tb.TadmaError):
        tb.eltwise(out, [out], [instr(Op.ADD, b=3)])
    with pytest.raises(tb.TadmaError):
        tb.eltwise(out, [out], [instr(99)])


# ---- copies through a transpose (tiled shared-memory path) -------------------

@pytest.mark.parametrize("shape,perm", [((70, 45), (1, 0)), ((3, 33, 100), (0, 2, 1)), ((2, 5, 37, 64), (0, 2, 3, 1)),
                                        ((4, 8, 96, 64), (0, 1, 3, 2)),
                                        # 16-byte aligned rows: the 64 x 64 vector tiles, with partial edge tiles
                                        ((3, 72, 136), (0, 2, 1)), ((200, 264), (1, 0)), ((2, 24, 16, 8), (0, 2, 3, 1)),
                                        # 16-bit: 64 x 256 pair-packed tiles (n_j >= 256), partial in both dims
                                        ((2, 520, 72), (0, 2, 1)), ((600, 136), (1, 0)), ((3, 264, 4, 16), (0, 2, 3, 1))])
@pytest.mark.parametrize("dt,out_dt", [(DType.F32, DType.F32), (DType.BF16, DType.BF16), (DType.F16, DType.F32),
                                       (DType.F16, DType.F16), (DType.F16, DType.BF16), (DType.BF16, DType.F16)])
def test_transpose_copy_and_cast(shape, perm, dt, out_dt):
    import torch
    x = gen(shape, dt, Dist.NORMAL, 0.0, 1.0, 30)
    xd = to_dev(x, dt)
    out_shape = [shape[p] for p in perm]
    strides = [xd.stride()[p] for p in perm]
    view = make_tensor(xd.data_ptr(), dt, out_shape, strides)  # x.permute(perm) as a strided view
    out = empty_dev(out_shape, out_dt)
    tb.eltwise(out, [view], [instr(Op.COPY)])
    torch.cuda.synchronize()
    ref = np.zeros(out_shape, dtype=from_dev(out).dtype)
    assert O.eltwise(ref, [np.transpose(x, perm)], [instr(Op.COPY)], out_dtype=out_dt, in_dtypes=[dt]) == 0
    assert np.array_equal(from_dev(out).view(np.uint8), ref.view(np.uint8))


def test_transpose64_with_chain():
    # aligned fp32 rows: the swizzled tile kernel runs the chain on the way out
    import torch
    x = gen((6, 136, 72), DType.F32, Dist.NORMAL, 0.0, 1.0, 32)
    xd = to_dev(x)
    view = make_tensor(xd.data_ptr(), DType.F32, [6, 72, 136], [136 * 72, 1, 72])
    out = empty_dev((6, 72, 136), DType.BF16)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=1.5), instr(Op.GELU)]
    tb.eltwise(out, [view], prog, Compute.F32)
    torch.cuda.synchronize()
    ref = np.zeros((6, 72, 136), np.uint16)
    assert O.eltwise(ref, [np.transpose(x, (0, 2, 1))], prog, Compute.F32, out_dtype=DType.BF16, in_dtypes=[DType.F32]) == 0
    assert ulp_diff(from_dev(out), ref, DType.BF16).max() <= 1


@pytest.mark.parametrize("n_j", [136, 520])
def test_transpose16_with_chain(n_j):
    # 16-bit in and out: the pair-packed tile kernel runs the chain on the way out
    import torch
    x = gen((3, n_j, 72), DType.BF16, Dist.NORMAL, 0.0, 1.0, 33)
    xd = to_dev(x, DType.BF16)
    view = make_tensor(xd.data_ptr(), DType.BF16, [3, 72, n_j], [n_j * 72, 1, 72])
    out = empty_dev((3, 72, n_j), DType.F16)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=1.5), instr(Op.GELU)]
    tb.eltwise(out, [view], prog, Compute.F32)
    torch.cuda.synchronize()
    ref = np.zeros((3, 72, n_j), np.uint16)
    assert O.eltwise(ref, [np.transpose(x, (0, 2, 1))], prog, Compute.F32, out_dtype=DType.F16, in_dtypes=[DType.BF16]) == 0
    assert ulp_diff(from_dev(out), ref, DType.F16).max() <= 1


def test_transpose_with_chain():
    import torch
    x = gen((6, 130, 66), DType.F32, Dist.NORMAL, 0.0, 1.0, 31)
    xd = to_dev(x)
    view = make_tensor(xd.data_ptr(), DType.F32, [6, 66, 130], [130 * 66, 1, 66])
    out = empty_dev((6, 66, 130), DType.BF16)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=1.5), instr(Op.GELU)]
    tb.eltwise(out, [view], prog, Compute.F32)
    torch.cuda.synchronize()
    ref = np.zeros((6, 66, 130), np.uint16)
    assert O.eltwise(ref, [np.transpose(x, (0, 2, 1))], prog, Compute.F32, out_dtype=DType.BF16, in_dtypes=[DType.F32]) == 0
    assert ulp_diff(from_dev(out), ref, DType.BF16).max() <= 1


# ---- narrow operands (raw-word vector kernel) -------------------------------
# Every input 1 or 2 bytes wide, or an innermost broadcast of at most 4 bytes:
# the kernel holds raw 16-byte words and converts at compute time.  Results
# must equal the oracle bit for bit (only exact ops in these chains).

@pytest.mark.parametrize("shape", [(64, 1024), (37, 1000), (3, 24), (5, 8)])
def test_narrow_operand_kinds(shape):
    R, C = shape
    x16 = gen(shape, DType.F16, Dist.NORMAL, 0, 1, 40)
    xb = gen(shape, DType.BF16, Dist.NORMAL, 0, 1, 41)
    u8 = gen(shape, DType.U8, Dist.INDEX, 0, 256, 42)
    i8 = (gen(shape, DType.I32, Dist.INDEX, 0, 256, 43) - 128).astype(np.int8)
    m = gen(shape, DType.F32, Dist.UNIFORM, -1, 1, 44) > 0
    # (m ? u8 : i8) + bf16: four narrow operands
    got, ref = run_both(shape, DType.F32, [(m, DType.BOOL), (u8, DType.U8), (i8, DType.I8), (xb, DType.BF16)],
                        [instr(Op.WHERE, b=1, c=2), instr(Op.ADD, b=3, round_dtype=DType.F32)])
    assert np.array_equal(got, ref)
    # f16 * u8 + i8 with a bool mask -> bool, u8, f16 outputs
    for odt in (DType.BOOL, DType.U8, DType.F16, DType.BF16, DType.I8):
        got, ref = run_both(shape, odt, [(x16, DType.F16), (u8, DType.U8), (i8, DType.I8)],
                            [instr(Op.MUL, b=1, round_dtype=DType.F32), instr(Op.ADD, b=2, round_dtype=DType.F32)])
        assert np.array_equal(got.view(np.uint8), ref.view(np.uint8)), odt
    # innermost-broadcast scalars of 4-byte types (f32, i32) next to narrow operands
    col_f = np.broadcast_to(gen((R, 1), DType.F32, Dist.NORMAL, 0, 1, 45), shape)
    col_i = np.broadcast_to(gen((R, 1), DType.I32, Dist.INDEX, 0, 100, 46), shape)
    got, ref = run_both(shape, DType.F32, [(x16, DType.F16), (col_f, DType.F32), (col_i, DType.I32)],
                        [instr(Op.MUL, b=1), instr(Op.SUB, b=2)])
    assert np.array_equal(got, ref)


def test_narrow_add_full_size_bits():
    # the same-shape 16-bit add at [8192, 8192]: every element checked
    import torch
    a = empty_dev((8192, 8192), DType.F16)
    b = empty_dev((8192, 8192), DType.F16)
    tb.fill(a, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=47)
    tb.fill(b, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=48)
    y = empty_dev((8192, 8192), DType.F16)
    tb.eltwise(y, [a, b], [instr(Op.ADD, b=1)])
    torch.cuda.synchronize()
    ref = (a.float() + b.float()).half()  # one fp32 add rounded once to fp16
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))


# ---- contiguous typed kernels (compile-time dtypes; single-op chains) -------

TYPED_OPS = [Op.ADD, Op.SUB, Op.MUL, Op.DIV, Op.RSUB, Op.RDIV, Op.MAX, Op.MIN]


@pytest.mark.parametrize("dt", [DType.F32, DType.F16, DType.BF16])
@pytest.mark.parametrize("op", TYPED_OPS)
def test_typed_single_op_bit_exact(dt, op):
    shape = (1000003,)  # odd: vector body + scalar tail
    a = gen(shape, dt, Dist.NORMAL, 0, 1, 50)
    b = gen(shape, dt, Dist.NORMAL, 1, 0.5, 51)
    got, ref = run_both(shape, dt, [(a, dt), (b, dt)], [instr(op, b=1, round_dtype=dt)])
    assert np.array_equal(got, ref), "tensor operand"
    got, ref = run_both((64, 1024), dt, [(a[:65536].reshape(64, 1024), dt)], [instr(op, b=SRC_IMM, imm=0.37)])
    assert np.array_equal(got, ref), "immediate"


@pytest.mark.parametrize("idt", [DType.F32, DType.F16, DType.BF16])
@pytest.mark.parametrize("odt", [DType.F32, DType.F16, DType.BF16])
def test_typed_casts_and_chains(idt, odt):
    shape = (4099, 24)
    a = gen(shape, idt, Dist.NORMAL, 0, 3, 52)
    b = gen(shape, idt, Dist.NORMAL, 0, 1, 53)
    got, ref = run_both(shape, odt, [(a, idt)], [])  # cast
    assert np.array_equal(got, ref)
    prog = [instr(Op.MUL, b=1, round_dtype=DType.F32), instr(Op.ADD, b=SRC_IMM, imm=0.5, round_dtype=DType.F32),
            instr(Op.RELU, round_dtype=DType.F32)]
    got, ref = run_both(shape, odt, [(a, idt), (b, idt)], prog)  # interpreted typed chain
    assert np.array_equal(got, ref)


def test_typed_strided_views():
    # typed kernels over folded rank > 1: a copy into a column slice (concat),
    # a batched permute that keeps the inner dim, an outer-dim broadcast add
    import torch
    src = gen((4, 40, 64), DType.F16, Dist.NORMAL, 0, 1, 54)
    big = torch.zeros((4, 100, 64), dtype=torch.float16, device="cuda")
    tb.eltwise(big[:, 60:], [to_dev(src)], [instr(Op.COPY)])
    torch.cuda.synchronize()
    got = from_dev(big)
    assert np.array_equal(got[:, 60:], src) and not got[:, :60].any()
    x = gen((3, 24, 5, 16), DType.BF16, Dist.NORMAL, 0, 1, 55)
    xd = to_dev(x, DType.BF16)
    y = empty_dev((3, 5, 24, 16), DType.BF16)
    tb.eltwise(y, [xd.permute(0, 2, 1, 3)], [instr(Op.COPY)])
    torch.cuda.synchronize()
    assert np.array_equal(from_dev(y), np.ascontiguousarray(x.transpose(0, 2, 1, 3)))
    a = gen((33, 40), DType.F32, Dist.NORMAL, 0, 1, 56)
    row = gen((1, 40), DType.F32, Dist.NORMAL, 0, 1, 57)
    for op in (Op.ADD, Op.MUL, Op.RSUB):
        got, ref = run_both((33, 40), DType.F32, [(a, DType.F32), (np.broadcast_to(row, (33, 40)), DType.F32)],
                            [instr(op, b=1)])
        assert np.array_equal(got, ref), op


@pytest.mark.parametrize("dt", [DType.F32, DType.F16, DType.BF16])
def test_typed_compare_and_where(dt):
    shape = (257, 40)
    a = gen(shape, dt, Dist.NORMAL, 0, 1, 58)
    b = gen(shape, dt, Dist.NORMAL, 0, 1, 59)
    b.reshape(-1)[::7] = a.reshape(-1)[::7]  # ties for EQ / LE / GE
    for op in (Op.EQ, Op.NE, Op.LT, Op.GT, Op.LE, Op.GE):
        got, ref = run_both(shape, DType.BOOL, [(a, dt), (b, dt)], [instr(op, b=1, round_dtype=DType.BOOL)])
        assert np.array_equal(got, ref), op
        got, ref = run_both(shape, DType.BOOL, [(a, dt)], [instr(op, b=SRC_IMM, imm=0.25)])
        assert np.array_equal(got, ref), op
    c = gen(shape, DType.F32, Dist.UNIFORM, -1, 1, 60) > 0
    got, ref = run_both(shape, dt, [(c, DType.BOOL), (a, dt), (b, dt)], [instr(Op.WHERE, b=1, c=2)])
    assert np.array_equal(got, ref)
    cu8 = gen(shape, DType.U8, Dist.INDEX, 0, 3, 61)  # 0 -> y, 1 or 2 -> x
    got, ref = run_both(shape, dt, [(cu8, DType.U8), (a, dt), (b, dt)], [instr(Op.WHERE, b=1, c=2)])
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("n_ins", [5, 6])
def test_five_and_six_operand_chains(n_ins):
    """Chains over up to TADMA_MAX_INPUTS = 6 operands (a LayerNorm with its
    affine parameters: x, mean, std, gamma, beta), broadcasts included;
    +, -, *, / round once, so the result is bit-exact against the oracle."""
    R, C = 96, 1024
    x = gen((R, C), DType.F32, Dist.NORMAL, 0.0, 1.0, 31)
    m = gen((R, 1), DType.F32, Dist.NORMAL, 0.0, 0.1, 32)
    s = gen((R, 1), DType.F32, Dist.UNIFORM, 0.5, 2.0, 33)
    g = gen((C,), DType.F32, Dist.NORMAL, 1.0, 0.02, 34)
    b = gen((C,), DType.F32, Dist.NORMAL, 0.0, 0.02, 35)
    c = gen((R, C), DType.F32, Dist.NORMAL, 0.0, 1.0, 36)
    ops = [x, m, s, g, b, c][:n_ins]
    prog = [instr(Op.SUB, b=1), instr(Op.DIV, b=2), instr(Op.MUL, b=3), instr(Op.ADD, b=4)]
    if n_ins == 6:
        prog.append(instr(Op.MUL, b=5))
    views, keep = [], []
    for a in ops:
        k, d = dev_view(np.broadcast_to(a, (R, C)), DType.F32)
        keep.append(k)
        views.append(d)
    out = empty_dev((R, C), DType.F32)
    tb.eltwise(out, views, prog, Compute.F32)
    ref = np.zeros((R, C), np.float32)
    assert O.eltwise(ref, [np.broadcast_to(a, (R, C)) for a in ops], prog, Compute.F32) == 0
    assert np.array_equal(from_dev(out), ref)
