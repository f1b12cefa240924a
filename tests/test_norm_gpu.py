"""Fused softmax / LayerNorm / RMSNorm vs the oracle (double-precision rows).

Tolerance: fp16/bf16 outputs within 1 ulp of the double result rounded to the
output type; fp32 outputs (row statistics accumulated in fp32) within the
north star's reduction bound, relative error <= 1e-5 * sqrt(L), measured
against max(|exact|, 1) for LayerNorm / RMSNorm outputs (values near 0) and
against |exact| for softmax (all outputs positive).
LayerNorm's ONNX form sqrt(var + eps) and the reference's std + eps
(Operations.hpp:205-220) are both checked; for var ~ 1 they differ by < 1e-5
relative, inside the fp16 tolerance.
"""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import Dist, DType, LNMode
from tests.helpers import as_f64, dev_view, empty_dev, from_dev, gen, to_dev, ulp_diff

pytestmark = pytest.mark.gpu

TOL = {DType.F16: 1, DType.BF16: 1}


def assert_close(got, ref, dt, L, softmax=False):
    if dt == DType.F32:
        scale = np.abs(ref.astype(np.float64)) if softmax else np.maximum(np.abs(ref.astype(np.float64)), 1.0)
        rel = np.abs(got.astype(np.float64) - ref) / scale
        assert rel.max() <= 1e-5 * np.sqrt(L), rel.max()
    else:
        d = ulp_diff(got, ref, dt)
        assert d.max() <= TOL[dt], d.max()


def _softmax_both(x, dt, axis):
    keep, xd = dev_view(x, dt)
    out = empty_dev(x.shape, dt)
    tb.softmax(xd, axis, out)
    ref = np.zeros(x.shape, dtype=from_dev(out).dtype)
    assert O.softmax(np.ascontiguousarray(x), axis, ref, dtype=dt) == 0
    return from_dev(out), ref


@pytest.mark.parametrize("dt,shape,axis", [
    (DType.F16, (5, 2048), -1),      # warp path, 8 chunks
    (DType.BF16, (7, 1024), -1),     # warp path, 4 chunks
    (DType.F32, (3, 7, 64), -1),     # warp path, 1 chunk (masked)
    (DType.F32, (9, 1000), -1),      # warp path, fp32
    (DType.BF16, (4, 1001), -1),     # L % 8 != 0 -> block path
    (DType.F16, (2, 5000), -1),      # long row -> block path
    (DType.F32, (4, 33, 16), 1),     # strided axis -> block path
])
def test_softmax(dt, shape, axis):
    x = gen(shape, dt, Dist.NORMAL, 0.0, 3.0, 1)
    got, ref = _softmax_both(x, dt, axis)
    assert_close(got, ref, dt, shape[axis], softmax=True)


def test_softmax_inplace_and_extremes():
    import torch
    x = gen((8, 2048), DType.F16, Dist.NORMAL, 0.0, 3.0, 2)
    x[0, :] = np.float16(11.5)           # exp(x) overflows fp16 without max subtraction
    x[1, 0] = np.float16(60000.0)
    xd = to_dev(x)
    tb.softmax(xd, -1, xd)
    torch.cuda.synchronize()
    ref = np.zeros_like(x)
    O.softmax(x, -1, ref)
    got = from_dev(xd)
    assert ulp_diff(got, ref, DType.F16).max() <= 1
    assert np.all(got[0] == np.float16(1.0 / 2048))
    assert got[1, 0] == np.float16(1.0)


def _ln_both(x, dt, g, b, gdt, eps, mode):
    kx, xd = dev_view(x, dt)
    gd = to_dev(g, gdt) if g is not None else None
    bd = to_dev(b, gdt) if b is not None else None
    out = empty_dev(x.shape, dt)
    tb.layer_norm(xd, -1, gd, bd, eps, out, mode)
    ref = np.zeros(x.shape, dtype=from_dev(out).dtype)
    assert O.layer_norm(np.ascontiguousarray(x), -1, g, b, eps, mode, ref, dtype=dt, gb_dtype=gdt) == 0
    return from_dev(out), ref


@pytest.mark.parametrize("mode", [LNMode.ONNX, LNMode.TADMA])
@pytest.mark.parametrize("dt,gdt,shape", [
    (DType.F16, DType.F16, (64, 1024)),   # config 4a row length, warp path with vector gamma/beta
    (DType.BF16, DType.BF16, (16, 2048)),
    (DType.F32, DType.F32, (8, 768)),     # BERT hidden size
    (DType.F16, DType.F32, (9, 1024)),    # gamma dtype differs -> scalar gamma loads
    (DType.F16, DType.F16, (3, 1000)),    # L % 8 != 0 -> block path
])
def test_layer_norm(mode, dt, gdt, shape):
    L = shape[-1]
    x = gen(shape, dt, Dist.NORMAL, 0.0, 1.0, 1)
    g = gen((L,), gdt, Dist.NORMAL, 1.0, 0.02, 2)
    b = gen((L,), gdt, Dist.NORMAL, 0.0, 0.02, 3)
    got, ref = _ln_both(x, dt, g, b, gdt, 1e-5, mode)
    assert_close(got, ref, dt, L)


def test_layer_norm_kat_alternating_rows():
    # KAT: a row of alternating +-1 has mean 0, std 1 -> y = +-gamma + beta (up to eps).
    L = 1024
    x = np.tile(np.array([1, -1], np.float16), (4, L // 2))
    got, ref = _ln_both(x, DType.F16, None, None, DType.F16, 0.0, LNMode.ONNX)
    assert np.array_equal(got, x) and np.array_equal(ref, x)


@pytest.mark.parametrize("dt,shape", [(DType.F16, (32, 1024)), (DType.F32, (5, 333)), (DType.BF16, (4, 4096))])
def test_rms_norm(dt, shape):
    x = gen(shape, dt, Dist.NORMAL, 0.0, 1.0, 4)
    kx, xd = dev_view(x, dt)
    out = empty_dev(shape, dt)
    tb.rms_norm(xd, -1, 0.0, out)
    ref = np.zeros(shape, dtype=from_dev(out).dtype)
    assert O.rms_norm(x, -1, 0.0, ref, dtype=dt) == 0
    assert_close(from_dev(out), ref, dt, shape[-1])


def test_config4_reduced_size():
    x = gen((2, 2048, 1024), DType.F16, Dist.NORMAL, 0.0, 1.0, 1)
    g = gen((1024,), DType.F16, Dist.NORMAL, 1.0, 0.02, 2)
    b = gen((1024,), DType.F16, Dist.NORMAL, 0.0, 0.02, 3)
    got, ref = _ln_both(x, DType.F16, g, b, DType.F16, 1e-5, LNMode.ONNX)
    assert ulp_diff(got, ref, DType.F16).max() <= 1
    s = gen((1, 2, 2048, 2048), DType.F16, Dist.NORMAL, 0.0, 3.0, 4)
    got, ref = _softmax_both(s, DType.F16, -1)
    assert ulp_diff(got, ref, DType.F16).max() <= 1


def test_config4_full_size_sampled():
    # Full config 4: LN [64, 2048, 1024] and softmax [32, 16, 2048, 2048] fp16,
    # inputs generated on the device; sampled rows checked against the oracle,
    # every softmax row checked to sum to 1 (fp16 tolerance).
    import torch
    x = empty_dev((64, 2048, 1024), DType.F16)
    g = empty_dev((1024,), DType.F16)
    b = empty_dev((1024,), DType.F16)
    tb.fill(x, Dist.NORMAL, 0.0, 1.0, 0, 1)
    tb.fill(g, Dist.NORMAL, 1.0, 0.02, 0, 2)
    tb.fill(b, Dist.NORMAL, 0.0, 0.02, 0, 3)
    y = empty_dev(x.shape, DType.F16)
    tb.layer_norm(x, -1, g, b, 1e-5, y, LNMode.ONNX)
    s = empty_dev((32, 16, 2048, 2048), DType.F16)
    tb.fill(s, Dist.NORMAL, 0.0, 3.0, 0, 4)
    sy = empty_dev(s.shape, DType.F16)
    tb.softmax(s, -1, sy)
    torch.cuda.synchronize()
    rows = torch.as_tensor(np.random.default_rng(1).integers(0, 64 * 2048, 256), device="cuda")
    xs, ys = from_dev(x.view(-1, 1024)[rows]), from_dev(y.view(-1, 1024)[rows])
    ref = np.zeros_like(xs)
    O.layer_norm(xs, -1, from_dev(g), from_dev(b), 1e-5, LNMode.ONNX, ref)
    assert ulp_diff(ys, ref, DType.F16).max() <= 1
    rows = torch.as_tensor(np.random.default_rng(2).integers(0, 32 * 16 * 2048, 256), device="cuda")
    xs, ys = from_dev(s.view(-1, 2048)[rows]), from_dev(sy.view(-1, 2048)[rows])
    ref = np.zeros_like(xs)
    O.softmax(xs, -1, ref)
    assert ulp_diff(ys, ref, DType.F16).max() <= 1
    row_sums = sy.view(-1, 2048).float().sum(dim=1)
    assert float((row_sums - 1).abs().max()) < 2e-2
    # The reference's softmax (exp, then divide by the sum; Operations.hpp:190-193)
    # overflows fp16 exp for x > 11.09.  N(0, 3) over 2^31 elements puts about
    # 2.3e5 values there (z > 3.70); every output stays finite here, and those
    # rows match the oracle like the others.
    hot = (s.view(-1, 2048) > 11.09).any(dim=1)
    n_hot = int(hot.sum())
    assert n_hot > 100_000, n_hot
    assert float(s.float().max()) > 15.0
    assert bool(torch.isfinite(sy).all())
    rows = torch.nonzero(hot).flatten()[:: max(1, n_hot // 128)][:128]
    xs, ys = from_dev(s.view(-1, 2048)[rows]), from_dev(sy.view(-1, 2048)[rows])
    ref = np.zeros_like(xs)
    O.softmax(xs, -1, ref)
    assert ulp_diff(ys, ref, DType.F16).max() <= 1
