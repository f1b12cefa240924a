"""tadma_b200_reduce_chain (a reduction of a fused element-wise chain, one
kernel) against the oracle's two-step composition: the chain into a
compute-type temporary (or_eltwise), then the reduction (or_reduce).  max /
min / argmax / argmin are bit-exact; sums within the fp32 reduction
tolerance 1e-5 * sqrt(n) (their association order differs)."""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, Op, Reduce, instr, make_tensor
from tests.helpers import dev_view, empty_dev, from_dev, gen, to_dev, ulp_diff

pytestmark = pytest.mark.gpu


def both(op, ins, in_dts, prog, axis, keep=True, compute=Compute.F32):
    """ins: numpy arrays already broadcast to the execution shape (views allowed)."""
    shape = np.broadcast_shapes(*[a.shape for a in ins])
    ax = axis % len(shape)
    oshape = tuple(1 if d == ax else s for d, s in enumerate(shape)) if keep else tuple(s for d, s in enumerate(shape) if d != ax)
    arg = op in (Reduce.ARGMAX, Reduce.ARGMIN)
    odt = DType.I64 if arg else (DType.F64 if compute == Compute.F64 else DType.F32)
    keep_alive, devs = [], []
    for a, dt in zip(ins, in_dts):
        k, d = dev_view(np.broadcast_to(a, shape), dt)
        keep_alive.append(k)
        devs.append(d)
    out = empty_dev(oshape, odt)
    tb.reduce_chain(op, devs, prog, axis, out, compute)
    # oracle: chain into a compute-type temporary, then reduce
    tmp_dt = DType.F64 if compute == Compute.F64 else DType.F32
    tmp = np.zeros(shape, np.float64 if tmp_dt == DType.F64 else np.float32)
    assert O.eltwise(tmp, [np.broadcast_to(a, shape) for a in ins], prog, compute, out_dtype=tmp_dt, in_dtypes=in_dts) == 0
    ref = np.zeros(oshape, np.int64 if arg else tmp.dtype)
    assert O.reduce(op, tmp, axis, ref) == 0
    return from_dev(out), ref, tmp


def close(got, ref, tmp, op, axis, max_ulp=0):
    """max_ulp: the chain's own fp32 error when it holds a transcendental op
    (CUDA's tanhf / expf are within 2 ulp of the oracle's correctly rounded
    values), which max / min carry through unchanged."""
    if op in (Reduce.ARGMAX, Reduce.ARGMIN):
        assert np.array_equal(got, ref), (op.name, got, ref)
        return
    if op in (Reduce.MAX, Reduce.MIN):
        if max_ulp == 0:
            assert np.array_equal(got, ref, equal_nan=True), (op.name, got, ref)
        else:
            assert ulp_diff(got, ref, DType.F32).max() <= max_ulp, (op.name, got, ref)
        return
    n = tmp.shape[axis]
    scale = np.maximum(np.abs(tmp.astype(np.float64)).sum(axis=axis, keepdims=True).reshape(ref.shape), 1.0)
    if op in (Reduce.MEAN, Reduce.RMS):
        scale = scale / n
    if op in (Reduce.SUMSQ, Reduce.RMS):
        scale = np.maximum((tmp.astype(np.float64) ** 2).sum(axis=axis, keepdims=True).reshape(ref.shape), 1.0)
        scale = scale / n if op == Reduce.RMS else scale
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64)) / scale
    assert err.max() <= 1e-5 * np.sqrt(n), (op.name, err.max())


def test_config1_in_one_kernel():
    # y = sum_last(exp(A + b)): the chain add-then-exp, reduced in the same kernel.
    A = gen((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 1)
    b = gen((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 2)
    prog = [instr(Op.ADD, b=1), instr(Op.EXP)]
    got, ref, tmp = both(Reduce.SUM, [A, b], [DType.F32, DType.F32], prog, -1, keep=False)
    close(got, ref, tmp, Reduce.SUM, -1)
    np.testing.assert_allclose(got, np.exp((A + b).astype(np.float64)).sum(-1), rtol=1e-5 * np.sqrt(128))


@pytest.mark.parametrize("op", list(Reduce))
@pytest.mark.parametrize("dt", [DType.F32, DType.BF16, DType.F16])
def test_ops_last_axis_vector_path(op, dt):
    # (x - m)^2-style chain over a contiguous axis with a broadcast row operand.
    x = gen((37, 1000), dt, Dist.NORMAL, 0.0, 1.0, 3)
    m = gen((37, 1), DType.F32, Dist.NORMAL, 0.0, 0.1, 4)
    prog = [instr(Op.SUB, b=1), instr(Op.MUL, b=SRC_IMM, imm=1.5)]
    got, ref, tmp = both(op, [x, m], [dt, DType.F32], prog, -1)
    close(got, ref, tmp, op, -1)


@pytest.mark.parametrize("axis", [0, 1, 2])
@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MAX, Reduce.ARGMIN, Reduce.MEAN])
def test_middle_and_leading_axes_scalar_path(axis, op):
    x = gen((6, 50, 33), DType.F32, Dist.UNIFORM, -1, 1, 5)
    y = gen((1, 50, 1), DType.F32, Dist.UNIFORM, -1, 1, 6)
    prog = [instr(Op.MUL, b=1), instr(Op.TANH)]
    got, ref, tmp = both(op, [x, y], [DType.F32, DType.F32], prog, axis, keep=(axis != 1))
    close(got, ref, tmp, op, axis, max_ulp=2)


def test_nan_and_ties_arg_kinds():
    x = np.zeros((4, 300), np.float32)
    x[0, [10, 200]] = 3.0
    x[1, 150] = np.nan
    x[2, :] = -1.0
    x[3, 299] = 5.0
    prog = [instr(Op.ADD, b=SRC_IMM, imm=1.0)]
    for op in (Reduce.ARGMAX, Reduce.ARGMIN, Reduce.MAX):
        got, ref, tmp = both(op, [x], [DType.F32], prog, -1)
        close(got, ref, tmp, op, -1)
    got, _, _ = both(Reduce.ARGMAX, [x], [DType.F32], prog, -1, keep=False)
    assert list(got) == [10, 150, 0, 299]


def test_f64_and_i64_compute():
    xi = gen((9, 40), DType.I64, Dist.INDEX, 0, 1000, 7)
    yi = gen((9, 40), DType.I64, Dist.INDEX, 0, 1000, 8)
    prog = [instr(Op.SUB, b=1)]
    out = empty_dev((9, 1), DType.I64)
    tb.reduce_chain(Reduce.SUM, [to_dev(xi), to_dev(yi)], prog, -1, out, Compute.I64)
    assert np.array_equal(from_dev(out)[:, 0], (xi - yi).sum(-1))
    xd = gen((9, 40), DType.F64, Dist.NORMAL, 0, 1, 9)
    got, ref, tmp = both(Reduce.SUM, [xd], [DType.F64], [instr(Op.EXP)], -1, compute=Compute.F64)
    np.testing.assert_allclose(got, ref, rtol=1e-12)


def test_full_size_row_sum_of_chain_matches_two_step():
    # X[32*4096, 4096] fp32 rows: sum(x * 0.5 + 1) in one kernel vs eltwise + reduce on the GPU.
    import torch
    x = torch.empty((4096, 4096), dtype=torch.float32, device="cuda")
    tb.fill(x, Dist.UNIFORM, -1.0, 1.0, 0, 1)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=0.5), instr(Op.ADD, b=SRC_IMM, imm=1.0)]
    fused = torch.empty((4096, 1), dtype=torch.float32, device="cuda")
    tb.reduce_chain(Reduce.SUM, [x], prog, -1, fused, Compute.F32)
    tmp = torch.empty_like(x)
    tb.eltwise(tmp, [x], prog, Compute.F32)
    two = torch.empty((4096, 1), dtype=torch.float32, device="cuda")
    tb.reduce(Reduce.SUM, tmp, -1, two)
    np.testing.assert_allclose(fused.cpu().numpy(), two.cpu().numpy(), rtol=1e-5 * 64, atol=1e-3)
    mx = torch.empty((4096, 1), dtype=torch.float32, device="cuda")
    tb.reduce_chain(Reduce.MAX, [x], prog, -1, mx, Compute.F32)
    mx2 = torch.empty_like(mx)
    tb.reduce(Reduce.MAX, tmp, -1, mx2)
    assert torch.equal(mx, mx2)


@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.ARGMAX, Reduce.MIN])
def test_vector_path_with_ragged_tail(op):
    # rows of 1003 inside a padded [4, 1008] buffer: 16-byte aligned rows, 125
    # vectors + a 3-element tail per row
    import torch
    full = gen((4, 1008), DType.F32, Dist.NORMAL, 0, 1, 10)
    xd = to_dev(full)
    view = make_tensor(xd.data_ptr(), DType.F32, [4, 1003], [1008, 1])
    prog = [instr(Op.ABS), instr(Op.SQRT)]
    arg = op == Reduce.ARGMAX
    out = empty_dev((4, 1), DType.I64 if arg else DType.F32)
    tb.reduce_chain(op, [view], prog, -1, out, Compute.F32)
    tmp = np.zeros((4, 1003), np.float32)
    assert O.eltwise(tmp, [full[:, :1003]], prog, Compute.F32, out_dtype=DType.F32, in_dtypes=[DType.F32]) == 0
    ref = np.zeros((4, 1), np.int64 if arg else np.float32)
    assert O.reduce(op, tmp, -1, ref) == 0
    close(from_dev(out), ref, tmp, op, -1)


# Operands that are one row for every output (a bias over the reduced axis),
# of the rows' dtype (the typed kernel) or another one (the interpreter).
@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MEAN, Reduce.MAX, Reduce.ARGMAX])
@pytest.mark.parametrize("xdt,bdt", [(DType.BF16, DType.F32), (DType.F32, DType.F32), (DType.F16, DType.BF16)])
def test_column_operand_staged_any_dtype(op, xdt, bdt):
    x = gen((37, 1000), xdt, Dist.NORMAL, 0.0, 1.0, 30)
    b = gen((1000,), bdt, Dist.NORMAL, 0.0, 1.0, 31)
    prog = [instr(Op.ADD, b=1), instr(Op.EXP)]
    got, ref, tmp = both(op, [x, b], [xdt, bdt], prog, -1)
    close(got, ref, tmp, op, -1, max_ulp=2)


def test_two_column_operands_and_ragged_rows():
    # rows of 1003 in a [33, 1008] buffer (16-byte aligned rows, a 3-element
    # tail), two column operands of other dtypes
    import torch
    full = gen((33, 1008), DType.F32, Dist.NORMAL, 0, 1, 32)
    xd = to_dev(full)
    view = make_tensor(xd.data_ptr(), DType.F32, [33, 1003], [1008, 1])
    b1 = gen((1003,), DType.F16, Dist.NORMAL, 0, 1, 33)
    b2 = gen((1003,), DType.BF16, Dist.UNIFORM, 0.5, 1.5, 34)
    k1, d1 = dev_view(np.broadcast_to(b1, (33, 1003)), DType.F16)
    k2, d2 = dev_view(np.broadcast_to(b2, (33, 1003)), DType.BF16)
    prog = [instr(Op.ADD, b=1), instr(Op.MUL, b=2), instr(Op.TANH)]
    for op in (Reduce.SUM, Reduce.MIN):
        out = empty_dev((33, 1), DType.F32)
        tb.reduce_chain(op, [view, d1, d2], prog, -1, out, Compute.F32)
        shape = (33, 1003)
        tmp = np.zeros(shape, np.float32)
        assert O.eltwise(tmp, [full[:, :1003], np.broadcast_to(b1, shape), np.broadcast_to(b2, shape)], prog,
                         Compute.F32, out_dtype=DType.F32, in_dtypes=[DType.F32, DType.F16, DType.BF16]) == 0
        ref = np.zeros((33, 1), np.float32)
        assert O.reduce(op, tmp, -1, ref) == 0
        close(from_dev(out), ref, tmp, op, -1, max_ulp=2)


# Chains of the row-operand form op1(x, m) -> [unary] -> [square], m one value
# per output row or an immediate: tadma_b200_reduce_chain runs them on the
# reduction engine's row kernel (reduce_rowop_kernel).
ROWOP_PROGS = {
    "variance": [instr(Op.SUB, b=1), instr(Op.POW, b=SRC_IMM, imm=2.0)],
    "softmax_denominator": [instr(Op.SUB, b=1), instr(Op.EXP)],
    "scaled": [instr(Op.MUL, b=SRC_IMM, imm=0.5)],
    "plain": [],
    "square": [instr(Op.POW, b=SRC_IMM, imm=2.0)],
    "ratio_abs": [instr(Op.DIV, b=1), instr(Op.ABS)],
}


@pytest.mark.parametrize("name", list(ROWOP_PROGS))
@pytest.mark.parametrize("op", list(Reduce))
@pytest.mark.parametrize("dt,shape", [(DType.F32, (37, 1000)), (DType.BF16, (37, 1000)), (DType.F16, (5, 1003))])
def test_row_operand_chains(name, op, dt, shape):
    prog = ROWOP_PROGS[name]
    x = gen(shape, dt, Dist.NORMAL, 0.0, 1.0, 11)
    ins, dts = [x], [dt]
    if any(i.b == 1 for i in prog):
        ins.append(gen((shape[0], 1), DType.F32, Dist.NORMAL, 0.5, 0.3, 12))
        dts.append(DType.F32)
    got, ref, tmp = both(op, ins, dts, prog, -1)
    # exp through CUDA's expf: max / min within its 2 ulp
    close(got, ref, tmp, op, -1, max_ulp=2 if name == "softmax_denominator" else 0)


def test_row_operand_chain_reaches_the_row_kernel():
    import torch
    from tests.test_dispatch_gpu import kernels_of
    x = torch.empty((256, 4096), dtype=torch.float32, device="cuda")
    tb.fill(x, Dist.NORMAL, 0.0, 1.0, 0, 13)
    m = torch.empty((256, 1), dtype=torch.float32, device="cuda")
    tb.fill(m, Dist.NORMAL, 0.0, 0.1, 0, 14)
    mv = make_tensor(m.data_ptr(), DType.F32, [256, 4096], [1, 0])
    out = torch.empty((256, 1), dtype=torch.float32, device="cuda")
    names = kernels_of(lambda: tb.reduce_chain(Reduce.MEAN, [x, mv], ROWOP_PROGS["variance"], -1, out, Compute.F32))
    assert "reduce_rowop_kernel" in names, names


POST = [instr(Op.ADD, b=SRC_IMM, imm=1e-5, round_dtype=DType.F32), instr(Op.SQRT, round_dtype=DType.F32)]


@pytest.mark.parametrize("name,axis", [("variance", -1), ("plain", -1), ("ratio_abs", -1), ("plain", 0)])
@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MEAN, Reduce.MAX, Reduce.RMS])
def test_post_chain(name, axis, op):
    """out = post(reduce(chain)): sqrt(reduced + 1e-5) applied before the
    store, in the row-operand kernel (last axis) and the general kernel
    (axis 0); the oracle applies the same post chain to its reduction."""
    prog = ROWOP_PROGS[name]
    x = gen((37, 1000), DType.F32, Dist.UNIFORM, 0.0, 2.0, 15)
    ins, dts = [x], [DType.F32]
    if any(i.b == 1 for i in prog):
        ins.append(gen((37, 1), DType.F32, Dist.NORMAL, 0.5, 0.3, 16))
        dts.append(DType.F32)
    shape = x.shape
    ax = axis % 2
    oshape = tuple(1 if d == ax else s for d, s in enumerate(shape))
    keep_alive, devs = [], []
    for a, dt in zip(ins, dts):
        k, d = dev_view(np.broadcast_to(a, shape), dt)
        keep_alive.append(k)
        devs.append(d)
    out = empty_dev(oshape, DType.F32)
    tb.reduce_chain(op, devs, prog, axis, out, Compute.F32, post=POST)
    tmp = np.zeros(shape, np.float32)
    assert O.eltwise(tmp, [np.broadcast_to(a, shape) for a in ins], prog, Compute.F32, out_dtype=DType.F32,
                     in_dtypes=dts) == 0
    red = np.zeros(oshape, np.float32)
    assert O.reduce(op, tmp, axis, red) == 0
    ref = np.zeros_like(red)
    assert O.eltwise(ref, [red], POST, Compute.F32) == 0
    got = from_dev(out)
    if op == Reduce.MAX:
        assert np.array_equal(got, ref)
    else:
        # the reduction's tolerance, halved by the square root
        assert np.all(np.abs(got.astype(np.float64) / ref - 1) <= 1e-5 * np.sqrt(shape[ax])), (op, name)


def test_post_chain_rejected_for_arg_ops():
    x = empty_dev((4, 64), DType.F32)
    out = empty_dev((4,), DType.I64)
    with pytest.raises(Exception):
        tb.reduce_chain(Reduce.ARGMAX, [x], [], -1, out, Compute.F32, post=POST)
