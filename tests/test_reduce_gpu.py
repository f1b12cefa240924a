"""Reductions (tadma_b200_reduce) vs the oracle (or_reduce, fp64 accumulation).

Tolerance (north star): fp32 |got - exact| <= 1e-5 * sqrt(n) * scale with
scale = max(|exact|, sum|x| / sqrt(n)) (a cancellation-aware relative error);
fp16/bf16 outputs <= 2e-2 relative (and <= 1 ulp of the output in practice);
max / min / argmax / argmin / integer sums are exact.
"""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import Dist, DType, Op, Reduce, make_tensor
from tests.helpers import as_f64, dev_view, empty_dev, from_dev, gen, to_dev

pytestmark = pytest.mark.gpu


def out_shape(shape, axis, keep):
    ax = axis % len(shape)
    s = list(shape)
    if keep:
        s[ax] = 1
    else:
        del s[ax]
    return s


def run_both(op, x, dt, axis, keep=True, out_dt=None, pre=Op.COPY):
    out_dt = out_dt if out_dt is not None else (DType.I64 if op in (Reduce.ARGMAX, Reduce.ARGMIN) else dt)
    keepalive, xd = dev_view(x, dt)
    oshape = out_shape(x.shape, axis, keep)
    out = empty_dev(oshape, out_dt)
    tb.reduce(op, xd, axis, out, pre)
    ref = np.zeros(oshape, dtype=from_dev(out).dtype)
    assert O.reduce(op, x, axis, ref, pre, x_dtype=dt, out_dtype=out_dt) == 0
    return from_dev(out), ref


def check_close(got, ref, x, dt, axis, op, out_dt):
    if op in (Reduce.MAX, Reduce.MIN, Reduce.ARGMAX, Reduce.ARGMIN) or not np.issubdtype(got.dtype, np.floating) and out_dt != DType.BF16:
        assert np.array_equal(got, ref), f"{op.name}: {(got != ref).sum()} mismatches"
        return
    g, r = as_f64(got, out_dt), as_f64(ref, out_dt)
    n = x.shape[axis % x.ndim]
    if out_dt == DType.F32:
        xs = np.abs(as_f64(np.ascontiguousarray(x), dt))
        if op in (Reduce.SUMSQ, Reduce.RMS):
            xs = xs * xs
        scale_sum = xs.sum(axis=axis, keepdims=g.ndim == x.ndim)
        if op in (Reduce.MEAN, Reduce.RMS):
            scale_sum = scale_sum / n
        scale = np.maximum(np.abs(r), scale_sum.reshape(r.shape) / np.sqrt(n))
        err = np.abs(g - r)
        assert np.all(err <= 1e-5 * np.sqrt(n) * scale + 1e-30), f"{op.name}: max rel {np.max(err / (scale + 1e-30))}"
    else:
        assert np.all(np.abs(g - r) <= 2e-2 * np.maximum(np.abs(r), 1e-3)), op.name


@pytest.mark.parametrize("shape", [(5, 33, 136), (5, 33, 130)])  # vector and scalar column paths
@pytest.mark.parametrize("dt", [DType.F32, DType.F16, DType.BF16])
@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MEAN, Reduce.MAX, Reduce.MIN, Reduce.ARGMAX, Reduce.ARGMIN,
                                Reduce.SUMSQ, Reduce.RMS])
@pytest.mark.parametrize("axis", [0, 1, 2, -1])
def test_reduce_axes(shape, dt, op, axis):
    x = gen(shape, dt, Dist.NORMAL, 0.0, 1.0, 3)
    out_dt = DType.I64 if op in (Reduce.ARGMAX, Reduce.ARGMIN) else dt
    got, ref = run_both(op, x, dt, axis, keep=True, out_dt=out_dt)
    check_close(got, ref, x, dt, axis, op, out_dt)


@pytest.mark.parametrize("axis", [0, 1, 2])
def test_reduce_keepdims_false_and_fp32_out_of_fp16(axis):
    x = gen((5, 33, 136), DType.F16, Dist.NORMAL, 0.0, 1.0, 4)
    got, ref = run_both(Reduce.SUM, x, DType.F16, axis, keep=False, out_dt=DType.F32)
    check_close(got, ref, x, DType.F16, axis, Reduce.SUM, DType.F32)


def test_config1_row_sum_of_exp():
    # Config 1: y = sum_{last}(exp(A + b)) -> [64]; the exp is fused as the reduction's pre-op.
    A = gen((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 1)
    b = gen((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 2)
    t = (A + b).astype(np.float32)
    got, ref = run_both(Reduce.SUM, t, DType.F32, -1, keep=False, pre=Op.EXP)
    check_close(got, ref, np.exp(t.astype(np.float64)), DType.F64, -1, Reduce.SUM, DType.F32)


def test_argmax_ties_and_nan():
    x = np.zeros((6, 300), np.float32)
    x[0, [7, 100, 299]] = 5.0                      # ties -> first
    x[1, :] = -np.inf                               # all -inf -> 0
    x[2, [50, 200]] = np.nan                        # NaN counts as max, first NaN
    x[3, 299] = 1.0
    x[4, 0] = 1.0
    x[5, 150:] = 2.0
    for op, want in ((Reduce.ARGMAX, [7, 0, 50, 299, 0, 150]), (Reduce.ARGMIN, [0, 0, 50, 0, 1, 0])):
        got, ref = run_both(op, x, DType.F32, -1, keep=False)
        assert list(got) == want and list(ref) == want, (op.name, got, ref)
        got, ref = run_both(op, np.ascontiguousarray(x.T), DType.F32, 0, keep=False)
        assert list(got) == want and list(ref) == want, (op.name, "col", got, ref)


def test_max_propagates_nan():
    x = gen((4, 100), DType.F32, Dist.NORMAL, 0, 1, 5)
    x[1, 50] = np.nan
    got, ref = run_both(Reduce.MAX, x, DType.F32, -1, keep=False)
    assert np.isnan(got[1]) and np.isnan(ref[1])
    assert np.array_equal(got[[0, 2, 3]], ref[[0, 2, 3]])


@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MEAN, Reduce.MAX, Reduce.ARGMAX])
def test_int64_generic_exact(op):
    x = gen((7, 50, 9), DType.I64, Dist.INDEX, 0, 1000, 6) - 500
    got, ref = run_both(op, x, DType.I64, 1, keep=True)
    assert np.array_equal(got, ref)


def test_strided_input_generic_path():
    base = gen((40, 64), DType.F32, Dist.NORMAL, 0, 1, 7)
    view = base[::2, ::3]  # non-foldable strides
    got, ref = run_both(Reduce.SUM, view, DType.F32, 1)
    check_close(got, ref, view, DType.F32, 1, Reduce.SUM, DType.F32)


@pytest.mark.parametrize("n", [1, 3, 31, 33, 4097, 70001])
def test_row_lengths(n):
    x = gen((3, n), DType.BF16, Dist.UNIFORM, -1, 1, n)
    for op in (Reduce.SUM, Reduce.ARGMAX):
        got, ref = run_both(op, x, DType.BF16, -1, keep=False, out_dt=DType.F32 if op == Reduce.SUM else DType.I64)
        check_close(got, ref, x, DType.BF16, -1, op, DType.F32 if op == Reduce.SUM else DType.I64)


def test_config3_reduced_size():
    # BASELINE config 3 shapes scaled down on the batch axis: X[2, 4096, 4096] ~ U(-1, 1).
    x = gen((2, 512, 4096), DType.F32, Dist.UNIFORM, -1.0, 1.0, 1)
    for op, axis in ((Reduce.SUM, -1), (Reduce.MAX, -1), (Reduce.ARGMAX, -1), (Reduce.MEAN, 1)):
        got, ref = run_both(op, x, DType.F32, axis, keep=op != Reduce.ARGMAX)
        check_close(got, ref, x, DType.F32, axis, op, DType.I64 if op == Reduce.ARGMAX else DType.F32)


def test_config3_full_size_sampled():
    # Full config 3: X[32, 4096, 4096] fp32 generated on the device; the oracle
    # checks 64 sampled (batch, row) pairs for the last-axis ops and 2 whole
    # batches for the middle-axis mean.
    import torch
    x = empty_dev((32, 4096, 4096), DType.F32)
    tb.fill(x, Dist.UNIFORM, -1.0, 1.0, seed=0, stream_id=1)
    outs = {}
    for op, axis, dt in ((Reduce.SUM, -1, DType.F32), (Reduce.MAX, -1, DType.F32), (Reduce.ARGMAX, -1, DType.I64),
                         (Reduce.MEAN, 1, DType.F32)):
        o = empty_dev(out_shape((32, 4096, 4096), axis, op != Reduce.ARGMAX), dt)
        tb.reduce(op, x, axis, o)
        outs[op] = o
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    bs, rs = rng.integers(0, 32, 64), rng.integers(0, 4096, 64)
    rows = from_dev(x[torch.as_tensor(bs, device="cuda"), torch.as_tensor(rs, device="cuda")])
    s = from_dev(outs[Reduce.SUM])[bs, rs, 0]
    m = from_dev(outs[Reduce.MAX])[bs, rs, 0]
    a = from_dev(outs[Reduce.ARGMAX])[bs, rs]
    exact = rows.astype(np.float64).sum(axis=1)
    assert np.all(np.abs(s - exact) <= 1e-5 * 64 * np.maximum(np.abs(exact), np.abs(rows).sum(1) / 64))
    assert np.array_equal(m, rows.max(axis=1))
    assert np.array_equal(a, rows.argmax(axis=1))
    for b in (0, 31):
        xb = from_dev(x[b])
        mean = from_dev(outs[Reduce.MEAN])[b, 0]
        exact = xb.astype(np.float64).mean(axis=0)
        assert np.all(np.abs(mean - exact) <= 1e-5 * 64 * np.maximum(np.abs(exact), np.abs(xb).mean(0) / 64))


def test_invalid():
    x = empty_dev((4, 8), DType.F32)
    with pytest.raises(tb.TadmaError):
        tb.reduce(Reduce.SUM, x, 2, empty_dev((4, 1), DType.F32))
    with pytest.raises(tb.TadmaError):
        tb.reduce(Reduce.ARGMAX, x, 1, empty_dev((4, 1), DType.F32))
    with pytest.raises(tb.TadmaError):
        tb.reduce(Reduce.SUM, x, 1, empty_dev((4, 2), DType.F32))


# ---- split-R (two-pass) paths: few outputs, long reduced axis ----------------

@pytest.mark.parametrize("dt", [DType.F32, DType.BF16])
@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MEAN, Reduce.MAX, Reduce.ARGMAX, Reduce.ARGMIN, Reduce.RMS])
def test_row_split_long_rows(dt, op):
    x = gen((3, 200003), dt, Dist.NORMAL, 0.0, 1.0, 21)  # odd length: vector body + scalar tail
    got, ref = run_both(op, x, dt, -1, keep=False, out_dt=DType.I64 if op in (Reduce.ARGMAX, Reduce.ARGMIN) else DType.F32)
    check_close(got, ref, x, dt, -1, op, DType.I64 if op in (Reduce.ARGMAX, Reduce.ARGMIN) else DType.F32)


def test_row_split_full_reduction_and_ties():
    n = 1 << 22
    x = gen((1, n), DType.F32, Dist.UNIFORM, -1, 1, 22)
    x[0, [123457, 2000001, 4000000]] = 7.0  # equal maxima in different chunks -> the first wins
    got, ref = run_both(Reduce.ARGMAX, x, DType.F32, -1, keep=False)
    assert got[0] == 123457 and ref[0] == 123457
    got, ref = run_both(Reduce.SUM, x, DType.F32, -1, keep=False, out_dt=DType.F32)
    check_close(got, ref, x, DType.F32, -1, Reduce.SUM, DType.F32)


@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MAX, Reduce.ARGMAX, Reduce.MEAN])
def test_col_split_long_axis(op):
    x = gen((2, 100000, 64), DType.F32, Dist.NORMAL, 0.0, 1.0, 23)
    out_dt = DType.I64 if op == Reduce.ARGMAX else DType.F32
    got, ref = run_both(op, x, DType.F32, 1, keep=op != Reduce.ARGMAX, out_dt=out_dt)
    check_close(got, ref, x, DType.F32, 1, op, out_dt)


def test_split_results_are_deterministic():
    import torch
    x = empty_dev((2, 1 << 21), DType.F32)
    tb.fill(x, Dist.NORMAL, 0, 1, 0, 24)
    a = empty_dev((2,), DType.F32)
    b = empty_dev((2,), DType.F32)
    tb.reduce(Reduce.SUM, x, -1, a)
    tb.reduce(Reduce.SUM, x, -1, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("shape", [(5, 4100), (3, 70000)])  # vector path with a tail; split-R path (few long rows)
def test_nan_inf_extremes_vector_paths(shape):
    R, L = shape
    x = gen(shape, DType.F32, Dist.UNIFORM, -1, 1, 21)
    x[0, 4000] = np.inf
    x[0, 4001] = np.nan          # NaN after +inf: NaN wins max, first NaN wins argmax
    x[1, :] = -np.inf
    x[1, L - 1] = np.nan         # NaN in the tail
    x[2, 3] = np.inf
    x[2, L - 2] = np.inf         # inf ties: first index
    if R > 3:
        x[3, 1024:1028] = np.nan  # a whole 16-byte vector of NaN
        x[4, 0] = -np.inf
    for op in (Reduce.MAX, Reduce.MIN, Reduce.ARGMAX, Reduce.ARGMIN):
        got, ref = run_both(op, x, DType.F32, -1, keep=False)
        if op in (Reduce.ARGMAX, Reduce.ARGMIN):
            assert np.array_equal(got, ref), (op.name, got, ref)
        else:
            assert np.array_equal(np.isnan(got), np.isnan(ref)), (op.name, got, ref)
            assert np.array_equal(got[~np.isnan(got)], ref[~np.isnan(ref)]), (op.name, got, ref)


@pytest.mark.parametrize("dt", [DType.F16, DType.BF16, DType.F32])
@pytest.mark.parametrize("pre", [Op.COPY, Op.EXP])
def test_arg_reductions_16bit_and_preop_vector_path(dt, pre):
    # 8-element (16-bit) and 4-element (fp32) vectors; ties inside one vector,
    # across vectors of one lane and across lanes; NaN; the pre-op applied in
    # the final in-vector search too.
    x = gen((6, 4096), dt, Dist.UNIFORM, -1, 1, 23)
    v = {DType.F16: np.float16(4.0).view(np.uint16), DType.BF16: np.uint16(0x4080), DType.F32: np.float32(4.0)}[dt]
    nan = {DType.F16: np.float16(np.nan).view(np.uint16), DType.BF16: np.uint16(0x7FC0), DType.F32: np.float32(np.nan)}[dt]
    x[0, [3, 5]] = v            # tie inside one vector -> 3
    x[1, [2000, 8, 300]] = v    # ties across lanes -> 8
    x[2, [4095, 1024]] = v      # -> 1024
    x[3, 77] = nan              # NaN -> 77
    x[4, [10, 11]] = nan        # first NaN -> 10
    for op in (Reduce.ARGMAX, Reduce.ARGMIN):
        got, ref = run_both(op, x, dt, -1, keep=False, pre=pre)
        assert np.array_equal(got, ref), (op.name, dt, pre, got, ref)
    got, _ = run_both(Reduce.ARGMAX, x, dt, -1, keep=False, pre=pre)
    assert list(got[:5]) == [3, 8, 1024, 77, 10]
