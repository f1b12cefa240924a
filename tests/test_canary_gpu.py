"""Out-of-bounds write detection without a memory checker: every kernel writes
its output into a view of a larger byte buffer whose GUARD bytes before and
after the view, and the padding at the end of each row when a row pitch is
given, hold a known pattern.  After the call those bytes must be unchanged,
the inputs must be unchanged, and the guarded output must equal, bit for
bit, the same call writing into a plain contiguous tensor.  Shapes are odd
(vector bodies with scalar tails, ragged last blocks, split reductions) so
that every kernel's bounds arithmetic is exercised."""
import numpy as np
import pytest

import tadma_b200 as tb
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, LNMode, Op, Reduce, instr, make_tensor

pytestmark = pytest.mark.gpu

GUARD = 4096
PATTERN = 0xA5


class Guarded:
    """An output tensor of `shape` / `dtype` (torch) inside a guarded byte
    buffer; `pitch` (elements) is the row stride, >= shape[-1]."""

    def __init__(self, shape, dtype, pitch=None):
        import torch
        self.shape = tuple(shape)
        self.elt = torch.empty((), dtype=dtype).element_size()
        self.cols = self.shape[-1] if self.shape else 1
        self.rows = int(np.prod(self.shape[:-1])) if len(self.shape) > 1 else 1
        self.pitch = self.cols if pitch is None else pitch
        assert self.pitch >= self.cols
        self.nbytes = self.rows * self.pitch * self.elt
        self.buf = torch.full((2 * GUARD + self.nbytes,), PATTERN, dtype=torch.uint8, device="cuda")
        body = self.buf[GUARD:GUARD + self.nbytes].view(dtype)
        strides, acc = [], 1
        for d in reversed(range(len(self.shape))):
            strides.append(acc)
            acc *= self.pitch if d == len(self.shape) - 1 else self.shape[d]
        self.t = body.as_strided(self.shape, tuple(reversed(strides)))

    def check(self):
        import torch
        torch.cuda.synchronize()
        b = self.buf.cpu().numpy()
        assert np.all(b[:GUARD] == PATTERN), "write before the output"
        assert np.all(b[GUARD + self.nbytes:] == PATTERN), "write after the output"
        if self.pitch > self.cols:
            rows = b[GUARD:GUARD + self.nbytes].reshape(self.rows, self.pitch * self.elt)
            assert np.all(rows[:, self.cols * self.elt:] == PATTERN), "write into the row padding"


def snapshot(*ts):
    return [t.clone() for t in ts]


def unchanged(ts, before):
    import torch
    torch.cuda.synchronize()
    for t, b in zip(ts, before):
        assert torch.equal(t.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8)), "an input was written"


def rand(shape, dtype, stream_id, lo=-2.0, hi=2.0):
    import torch
    t = torch.empty(shape, dtype=dtype, device="cuda")
    tb.fill(t, Dist.UNIFORM, lo, hi, seed=7, stream_id=stream_id)
    return t


def same_bits(a, b):
    import torch
    torch.cuda.synchronize()
    assert torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


# ---- element-wise chains ------------------------------------------------------

@pytest.mark.parametrize("shape,dt,pitch", [
    ((37, 1000), "bfloat16", None), ((37, 1000), "bfloat16", 1008), ((3, 24), "bfloat16", None),
    ((1, 1), "bfloat16", None), ((129, 33), "bfloat16", 40)])
def test_affine_rows(shape, dt, pitch):
    import torch
    tdt = getattr(torch, dt)
    x, bias = rand(shape, tdt, 1), rand(shape[-1:], tdt, 2)
    before = snapshot(x, bias)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
            instr(Op.GELU, round_dtype=DType.F32)]
    bview = make_tensor(bias.data_ptr(), tb.torch_dtype_code(bias), list(shape), [0, 1])
    g = Guarded(shape, tdt, pitch)
    tb.eltwise(g.t, [x, bview], prog, Compute.F32)
    plain = torch.empty(shape, dtype=tdt, device="cuda")
    tb.eltwise(plain, [x, bview], prog, Compute.F32)
    g.check()
    unchanged([x, bias], before)
    same_bits(g.t, plain)


@pytest.mark.parametrize("shape,dt,pitch", [
    ((3, 5, 7), "float32", None), ((3, 5, 7), "float32", 8), ((129, 33), "float16", 40), ((7,), "float32", None),
    ((2, 1000003), "float32", None)])
def test_chain(shape, dt, pitch):
    import torch
    tdt = getattr(torch, dt)
    a, b = rand(shape, tdt, 3), rand(shape, tdt, 4)
    before = snapshot(a, b)
    prog = [instr(Op.ADD, b=1), instr(Op.EXP), instr(Op.MUL, b=SRC_IMM, imm=0.25)]
    g = Guarded(shape, tdt, pitch)
    tb.eltwise(g.t, [a, b], prog, Compute.F32)
    plain = torch.empty(shape, dtype=tdt, device="cuda")
    tb.eltwise(plain, [a, b], prog, Compute.F32)
    g.check()
    unchanged([a, b], before)
    same_bits(g.t, plain)


@pytest.mark.parametrize("shape", [(33, 65), (2, 31, 97), (64, 64), (72, 136), (3, 200, 264)])
def test_transpose(shape):
    import torch
    x = rand(shape, torch.float32, 5)
    before = snapshot(x)
    xt = x.transpose(-1, -2)
    g = Guarded(tuple(xt.shape), torch.bfloat16)
    tb.eltwise(g.t, [xt], [instr(Op.TANH)], Compute.F32)
    plain = torch.empty(tuple(xt.shape), dtype=torch.bfloat16, device="cuda")
    tb.eltwise(plain, [xt], [instr(Op.TANH)], Compute.F32)
    g.check()
    unchanged([x], before)
    same_bits(g.t, plain)


@pytest.mark.parametrize("shape", [(72, 136), (3, 200, 264), (2, 520, 72)])
@pytest.mark.parametrize("raw", [True, False])
def test_transpose16(shape, raw):
    # 16-bit in and out: pair-packed tiles, a plain copy (raw words) or a chain
    import torch
    x = rand(shape, torch.float16, 6)
    before = snapshot(x)
    xt = x.transpose(-1, -2)
    odt = torch.float16 if raw else torch.bfloat16
    prog = [instr(Op.COPY)] if raw else [instr(Op.TANH)]
    g = Guarded(tuple(xt.shape), odt)
    tb.eltwise(g.t, [xt], prog, Compute.F32)
    plain = torch.empty(tuple(xt.shape), dtype=odt, device="cuda")
    tb.eltwise(plain, [xt], prog, Compute.F32)
    g.check()
    unchanged([x], before)
    same_bits(g.t, plain)
    if raw:
        assert torch.equal(plain.view(torch.int16), xt.contiguous().view(torch.int16))


# ---- reductions -----------------------------------------------------------------

@pytest.mark.parametrize("shape,axis", [((37, 1001), -1), ((37, 1001), 0), ((3, 777, 65), 1),
                                        ((3, 200003), -1), ((2, 100000, 64), 1), ((5,), 0)])
@pytest.mark.parametrize("op", [Reduce.SUM, Reduce.MAX, Reduce.ARGMAX, Reduce.MEAN])
def test_reduce(shape, axis, op):
    import torch
    x = rand(shape, torch.float32, 6)
    before = snapshot(x)
    oshape = tuple(1 if d == axis % len(shape) else s for d, s in enumerate(shape))
    odt = torch.int64 if op == Reduce.ARGMAX else torch.float32
    g = Guarded(oshape, odt)
    tb.reduce(op, x, axis, g.t)
    plain = torch.empty(oshape, dtype=odt, device="cuda")
    tb.reduce(op, x, axis, plain)
    g.check()
    unchanged([x], before)
    same_bits(g.t, plain)


@pytest.mark.parametrize("shape,op", [((64, 128), Reduce.SUM), ((5, 3001), Reduce.MAX), ((7, 4099), Reduce.ARGMIN),
                                      ((3, 65), Reduce.SUM)])
def test_reduce_chain(shape, op):
    import torch
    a, b = rand(shape, torch.float16, 8), rand(shape[-1:], torch.float16, 9)
    before = snapshot(a, b)
    bview = make_tensor(b.data_ptr(), DType.F16, list(shape), [0, 1])
    prog = [instr(Op.ADD, b=1), instr(Op.EXP)]
    oshape = shape[:-1] + (1,)
    odt = torch.int64 if op == Reduce.ARGMIN else torch.float32
    g = Guarded(oshape, odt)
    tb.reduce_chain(op, [a, bview], prog, -1, g.t, Compute.F32)
    plain = torch.empty(oshape, dtype=odt, device="cuda")
    tb.reduce_chain(op, [a, bview], prog, -1, plain, Compute.F32)
    g.check()
    unchanged([a, b], before)
    same_bits(g.t, plain)


# ---- row normalisations ---------------------------------------------------------

@pytest.mark.parametrize("shape,dt,pitch", [((37, 1000), "float16", None), ((37, 1000), "float16", 1008),
                                            ((37, 999), "float16", 1000), ((5, 4096), "bfloat16", None),
                                            ((3, 7), "float32", None), ((2, 3, 2048), "float16", None)])
@pytest.mark.parametrize("kind", ["softmax", "layer_norm", "rms_norm"])
def test_row_norms(shape, dt, pitch, kind):
    import torch
    tdt = getattr(torch, dt)
    x = rand(shape, tdt, 10)
    gamma, beta = rand(shape[-1:], tdt, 11, 0.5, 1.5), rand(shape[-1:], tdt, 12)
    before = snapshot(x, gamma, beta)

    def run(out):
        if kind == "softmax":
            tb.softmax(x, -1, out)
        elif kind == "layer_norm":
            tb.layer_norm(x, -1, gamma, beta, 1e-5, out, LNMode.ONNX)
        else:
            tb.rms_norm(x, -1, 1e-6, out)

    g = Guarded(shape, tdt, pitch)
    run(g.t)
    plain = torch.empty(shape, dtype=tdt, device="cuda")
    run(plain)
    g.check()
    unchanged([x, gamma, beta], before)
    same_bits(g.t, plain)


# ---- gather ---------------------------------------------------------------------

@pytest.mark.parametrize("B,S,D,with_pos", [(5, 7, 72, True), (2, 9, 4096, True), (3, 5, 13, False), (1, 1, 8, True)])
def test_gather(B, S, D, with_pos):
    import torch
    V = 101
    table = rand((V, D), torch.float16, 13)
    pos = rand((S, D), torch.bfloat16, 14)
    ids = torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(3)).cuda()
    before = snapshot(table, pos, ids)
    add = make_tensor(pos.data_ptr(), DType.BF16, [B, S, D], [0, D, 1]) if with_pos else None
    g = Guarded((B, S, D), torch.bfloat16)
    tb.gather(table, 0, ids, g.t, add=add)
    plain = torch.empty((B, S, D), dtype=torch.bfloat16, device="cuda")
    tb.gather(table, 0, ids, plain, add=add)
    g.check()
    unchanged([table, pos, ids], before)
    same_bits(g.t, plain)


# ---- fill -------------------------------------------------------------------------

@pytest.mark.parametrize("shape,dt,pitch", [((37, 1001), "float32", None), ((37, 1001), "float32", 1004),
                                            ((5, 3), "bfloat16", 8), ((1,), "float16", None)])
def test_fill(shape, dt, pitch):
    import torch
    tdt = getattr(torch, dt)
    g = Guarded(shape, tdt, pitch)
    tb.fill(g.t, Dist.NORMAL, 0.0, 1.0, seed=1, stream_id=2)
    plain = torch.empty(shape, dtype=tdt, device="cuda")
    tb.fill(plain, Dist.NORMAL, 0.0, 1.0, seed=1, stream_id=2)
    g.check()
    same_bits(g.t, plain)
