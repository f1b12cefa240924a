"""Empty and degenerate inputs through every entry point, GPU against the
oracle: the same status code, no write to an empty output, the sums' identity
for an empty reduced axis, single-element rows, rank-0 tensors."""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, LNMode, Op, Reduce, Status, instr
from tests.helpers import empty_dev, from_dev, gen, to_dev, ulp_diff

pytestmark = pytest.mark.gpu


def _status(fn):
    try:
        fn()
        return 0
    except tb.TadmaError as e:
        return e.code


@pytest.mark.parametrize("shape", [(0,), (0, 16), (5, 0, 3)])
def test_eltwise_empty(shape):
    x = empty_dev(shape, DType.F32)
    y = empty_dev(shape, DType.F32)
    tb.eltwise(y, [x], [instr(Op.EXP)], Compute.F32)
    assert from_dev(y).size == 0


@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.SUMSQ, Reduce.MEAN, Reduce.MAX, Reduce.MIN, Reduce.ARGMAX])
def test_reduce_over_empty_axis(op):
    xh = np.zeros((4, 0), np.float32)
    out_dt = DType.I64 if op == Reduce.ARGMAX else DType.F32
    out = empty_dev((4, 1), out_dt)
    out.fill_(7)
    code = _status(lambda: tb.reduce(op, to_dev(xh), -1, out))
    ref = np.full((4, 1), 7, np.int64 if op == Reduce.ARGMAX else np.float32)
    rc = O.reduce(op, xh, -1, ref)
    assert code == rc
    if rc == 0:
        assert np.array_equal(from_dev(out), ref) and not ref.any()  # identity of the sums
    else:
        assert code == Status.ERR_INVALID and np.all(from_dev(out) == 7)  # nothing written


def test_reduce_to_empty_output_and_single_elements():
    out = empty_dev((0, 1), DType.F32)
    tb.reduce(Reduce.MAX, empty_dev((0, 9), DType.F32), -1, out)   # no rows: no-op
    x = gen((6, 1), DType.F32, Dist.NORMAL, 0, 1, 3)
    for op in (Reduce.SUM, Reduce.MAX, Reduce.ARGMIN, Reduce.MEAN):
        dt = DType.I64 if op == Reduce.ARGMIN else DType.F32
        o = empty_dev((6, 1), dt)
        tb.reduce(op, to_dev(x), -1, o)
        ref = np.zeros((6, 1), np.int64 if op == Reduce.ARGMIN else np.float32)
        assert O.reduce(op, x, -1, ref) == 0
        assert np.array_equal(from_dev(o), ref), op.name


def test_row_ops_on_empty_and_single_element_rows():
    for shape in ((0, 1024), (3, 0, 64)):
        x = empty_dev(shape, DType.F16)
        y = empty_dev(shape, DType.F16)
        tb.softmax(x, -1, y)
        tb.layer_norm(x, -1, None, None, 1e-5, y, LNMode.ONNX)
    x = gen((5, 1), DType.F16, Dist.NORMAL, 0, 1, 5)
    y = empty_dev((5, 1), DType.F16)
    tb.softmax(to_dev(x), -1, y)
    assert np.all(from_dev(y) == np.float16(1.0))  # softmax of one element
    tb.layer_norm(to_dev(x), -1, None, None, 1e-5, y, LNMode.ONNX)
    ref = np.zeros_like(x)
    assert O.layer_norm(x, -1, None, None, 1e-5, LNMode.ONNX, ref) == 0
    assert np.array_equal(from_dev(y), ref)  # (x - mean) = 0 exactly


def test_gather_empty_ids_and_empty_table():
    table = to_dev(gen((10, 64), DType.F16, Dist.NORMAL, 0, 1, 6))
    out = empty_dev((0, 64), DType.F16)
    tb.gather(table, 0, empty_dev((0,), DType.I64), out)        # no ids: no-op
    empty_table = empty_dev((0, 64), DType.F16)
    out2 = empty_dev((3, 64), DType.F16)
    ids = to_dev(np.array([0, 0, 0], np.int64))
    assert _status(lambda: tb.gather(empty_table, 0, ids, out2)) == Status.ERR_INVALID
    assert tb.error_flags(clear=True) == 0


@pytest.mark.parametrize("dt", [DType.F16, DType.BF16])
def test_layer_norm_large_mean_and_constant_rows(dt):
    # Rows far from zero mean, and constant rows (every x equals the mean):
    # the output next to 0 must be 0 or within 1 ulp of the exact value.
    L = 1024
    x = gen((8, L), DType.F32, Dist.NORMAL, 0.0, 1.0, 7)
    x[:4] += 1000.0
    x[4:6] = 3.0                      # constant rows -> exactly 0
    if dt == DType.F16:
        xs = x.astype(np.float16)
    else:  # bf16 bits (truncated fp32)
        xs = (np.frombuffer(x.astype(np.float32).tobytes(), np.uint32) >> 16).astype(np.uint16).reshape(8, L)
    y = empty_dev((8, L), dt)
    tb.layer_norm(to_dev(xs, dt), -1, None, None, 1e-5, y, LNMode.ONNX)
    ref = np.zeros_like(xs)
    assert O.layer_norm(xs, -1, None, None, 1e-5, LNMode.ONNX, ref, dtype=dt) == 0
    got = from_dev(y)
    assert ulp_diff(got, ref, dt).max() <= 1
    assert not got[4:6].astype(np.float32).any() if dt == DType.F16 else not (got[4:6] & 0x7FFF).any()


# ---- index widths: 32-bit index walks where they fit, 64-bit beyond ---------------

def test_strided_view_with_offsets_past_2_31():
    # Elements < 2^32 but an input offset >= 2^31: 32-bit quotients, 64-bit offsets.
    import torch
    base = torch.empty((2 ** 31 + 1024,), dtype=torch.float16, device="cuda")
    rows = torch.randn((2, 1024), device="cuda").to(torch.float16)
    view = base.as_strided((2, 1024), (2 ** 31, 1))
    view.copy_(rows)
    out = torch.empty((2, 1024), dtype=torch.float16, device="cuda")
    tb.eltwise(out, [view], [instr(Op.COPY)])
    out2 = torch.empty((2, 1024), dtype=torch.float32, device="cuda")
    tb.eltwise(out2, [view], [instr(Op.MUL, b=SRC_IMM, imm=2.0)], Compute.F32)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), rows.view(torch.int16))
    assert torch.equal(out2, rows.float() * 2)
    del base


def test_broadcast_past_2_32_elements():
    # More than 2^32 output elements: the 64-bit index walk.
    import torch
    rows = 2 ** 32 // 1024 + 3
    row = torch.arange(1024, device="cuda", dtype=torch.int32).to(torch.uint8)
    out = torch.empty((rows, 1024), dtype=torch.uint8, device="cuda")
    tb.eltwise(out, [row.expand(rows, 1024)], [instr(Op.COPY)])
    torch.cuda.synchronize()
    for r in (0, 1, 2 ** 22 - 1, 2 ** 22, rows - 1):
        assert torch.equal(out[r], row), r
    assert bool((out[-4:] == row).all())
    del out
