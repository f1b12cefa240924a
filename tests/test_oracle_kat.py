"""The CPU oracle against the analytic known-answer vectors in tests/golden
(pure-Python values, tests/golden/make_kats.py) and against numpy where numpy
implements the same IEEE operation.  Parity with the reference itself is
unpinned: it cannot be built here and ships no expected outputs."""
import ctypes
import json
import math
import os
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, LNMode, Op, Reduce, bf16_bits_to_f32, f32_to_bf16_bits, instr

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "kats.json")))
sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_kats import draw as KATS_DRAW  # noqa: E402  (pure-Python generator definition)
from make_kats import key as KATS_KEY  # noqa: E402


def unary_f64(op, xs):
    x = np.array(xs, np.float64)
    out = np.zeros_like(x)
    assert O.eltwise(out, [x], [instr(op)], Compute.F64) == 0
    return out


@pytest.mark.parametrize("name,op", [("gelu", Op.GELU), ("sigmoid", Op.SIGMOID), ("tanh", Op.TANH), ("exp", Op.EXP)])
def test_unary_kats(name, op):
    xs, want = zip(*KATS[name])
    got = unary_f64(op, xs)
    np.testing.assert_allclose(got, want, rtol=1e-13, atol=1e-300)


def test_gelu_equals_reference_expression_where_it_is_accurate():
    xs, want = zip(*KATS["gelu_reference_expr"])
    np.testing.assert_allclose(unary_f64(Op.GELU, xs), want, rtol=1e-12)


def test_map_to_shape():
    for dims, idx, want in KATS["map_to_shape"]:
        assert O.map_to_shape(dims, idx) == want


def test_generator_golden_values():
    a = O.fill((16,), DType.F32, Dist.NORMAL, 0.0, 1.0, 0, 1)
    assert np.array_equal(a, np.array(KATS["gen_normal_f32_seed0_sid1"], np.float32))
    a = O.fill((8,), DType.F32, Dist.NORMAL, 1.0, 0.02, 7, 11)
    assert np.array_equal(a, np.array(KATS["gen_normal_f32_seed7_sid11_p1_0.02"], np.float32))
    a = O.fill((16,), DType.F32, Dist.UNIFORM, -1.0, 1.0, 0, 1)
    assert np.array_equal(a, np.array(KATS["gen_uniform_f32_seed0_sid1"], np.float32))
    a = O.fill((16,), DType.I64, Dist.INDEX, 0, 50257, 0, 2)
    assert list(a) == KATS["gen_index_seed0_sid2_v50257"]


def _normal_cdf(x):
    return 0.5 * (1.0 + np.vectorize(math.erf)(x / math.sqrt(2.0)))


def test_generator_is_normal_and_shards():
    """NORMAL is a true N(p0, p1): moments, tail mass beyond 3 and 4 sigma, and
    the Kolmogorov-Smirnov distance against the normal CDF; an offset shard
    equals the rows it covers; fp16 / bf16 are the double value rounded once."""
    n = 1 << 20
    z = O.fill((n,), DType.F64, Dist.NORMAL, 0.0, 1.0, 0, 1)
    assert abs(z.mean()) < 5e-3 and abs(z.std() - 1) < 5e-3
    for k, p in ((3.0, 2.6998e-3), (4.0, 6.334e-5)):
        count, want = int((np.abs(z) > k).sum()), p * n
        assert abs(count - want) < 6 * math.sqrt(want), (k, count, want)
    zs = np.sort(z[:1 << 18])
    ecdf = np.arange(1, zs.size + 1) / zs.size
    assert np.abs(ecdf - _normal_cdf(zs)).max() < 1.63 / math.sqrt(zs.size) * 1.5
    assert np.abs(z).max() < 8.6  # u1 >= 2^-53 bounds |z| by sqrt(106 ln 2)
    a = O.fill((512, 1024), DType.F64, Dist.NORMAL, 0.0, 1.0, 0, 1)
    b = O.fill((256, 1024), DType.F64, Dist.NORMAL, 0.0, 1.0, 0, 1, offset=256 * 1024)
    assert np.array_equal(b, a[256:])
    with np.errstate(over="ignore"):
        h = O.fill((512, 1024), DType.F16, Dist.NORMAL, 0.0, 3.0, 0, 1)
        d = O.fill((512, 1024), DType.F64, Dist.NORMAL, 0.0, 3.0, 0, 1)
        assert np.array_equal(h, d.astype(np.float16))  # numpy rounds float64 -> float16 once
        f = O.fill((512, 1024), DType.F32, Dist.NORMAL, 0.0, 3.0, 0, 1)
        assert np.array_equal(f, d.astype(np.float32))
    bf = O.fill((4096,), DType.BF16, Dist.NORMAL, 0.0, 3.0, 0, 1)
    d = O.fill((4096,), DType.F64, Dist.NORMAL, 0.0, 3.0, 0, 1)
    assert [int(v) for v in bf] == [_bf16_exact(float(v)) for v in d]
    u = O.fill((512, 1024), DType.F32, Dist.UNIFORM, -1.0, 1.0, 0, 2)
    assert u.min() >= -1 and u.max() < 1 and abs(u.var() - 1 / 3) < 5e-3


def test_generator_matches_libm_box_muller():
    """The series ln / cos of the generator agree with libm's to ~1e-13."""
    k = KATS_KEY(0, 1)
    got = O.fill((4096,), DType.F64, Dist.NORMAL, 0.0, 1.0, 0, 1)
    for g in range(4096):
        u1 = float((KATS_DRAW(k, g, 0) >> 11) + 1) * 2.0 ** -53
        t = float(KATS_DRAW(k, g, 1) >> 11) * 2.0 ** -53
        want = math.sqrt(-2.0 * math.log(u1)) * math.cos(2.0 * math.pi * t)
        assert abs(got[g] - want) <= 1e-12 * max(1.0, abs(want))


def _bf16_exact(v):
    """Round a double to bf16 bits with exact rational arithmetic (ties to even)."""
    from fractions import Fraction
    if v != v:
        return None
    sign = 0x8000 if math.copysign(1.0, v) < 0 else 0
    a = Fraction(abs(v))
    if a == 0:
        return sign
    top = Fraction(2) ** 127 * (2 - Fraction(1, 256))
    if a >= top:
        return sign | 0x7F80
    E = max(math.floor(math.log2(abs(v))), -126)
    while Fraction(2) ** E > a and E > -126:
        E -= 1
    while Fraction(2) ** (E + 1) <= a:
        E += 1
    scaled = a / Fraction(2) ** (E - 7)
    m = math.floor(scaled)
    rem = scaled - m
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and m % 2 == 1):
        m += 1
    return sign | (((E + 127) << 7) + m - 128)


def test_double_to_16bit_rounds_once():
    """or_f64_to_f16 equals numpy's float64 -> float16 cast; or_f64_to_bf16 the
    exact rounding, on values whose fp32 detour would round twice."""
    rng = np.random.default_rng(3)
    L = O.lib()
    L.or_f64_to_f16.argtypes = [ctypes.c_double]
    L.or_f64_to_f16.restype = ctypes.c_uint16
    L.or_f64_to_bf16.argtypes = [ctypes.c_double]
    L.or_f64_to_bf16.restype = ctypes.c_uint16
    # halfway points of fp16 / bf16 nudged by one double ulp (the fp32 detour rounds them to the tie)
    h = rng.standard_normal(4000).astype(np.float16).astype(np.float64)
    ulp16 = np.spacing(h.astype(np.float16)).astype(np.float64)
    ties = h + ulp16 / 2
    x = np.concatenate([rng.standard_normal(4000) * 3e4, np.nextafter(ties, np.inf), np.nextafter(ties, -np.inf),
                        [65504.0, 65519.99999, 65520.0, 6e-8, 2.9802322387695312e-08, 2.98e-8, -0.0, 1e-300, np.inf,
                         -np.inf]])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    got = np.array([L.or_f64_to_f16(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, want)
    bx = np.concatenate([rng.standard_normal(3000) * 1e3, [3.0e38, 3.4e38, 1e-39, 9.2e-41, -0.0, 1.0 + 2.0 ** -8 + 2.0 ** -40,
                                                         1.0 + 2.0 ** -8 - 2.0 ** -40, 1.0 + 2.0 ** -8]])
    got = [int(L.or_f64_to_bf16(float(v))) for v in bx]
    assert got == [_bf16_exact(float(v)) for v in bx]


def test_conversions_match_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * np.float32(3e4),
                        np.array([65504, 65519.996, 65520, 6e-8, 3e-8, 2.98e-8, -0.0, np.inf, -np.inf], np.float32)])
    L = O.lib()
    f16 = np.array([L.or_f32_to_f16(float(v)) for v in x], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(f16, x.astype(np.float16).view(np.uint16))
    bf = np.array([L.or_f32_to_bf16(float(v)) for v in x], np.uint16)
    assert np.array_equal(bf, f32_to_bf16_bits(x))
    assert np.array_equal(bf16_bits_to_f32(bf)[:100], np.array([L.or_bf16_to_f32(int(h)) for h in bf[:100]], np.float32))


def test_elementwise_exact_ops_match_numpy():
    a = O.fill((64, 130), DType.F32, Dist.NORMAL, 0, 1, 0, 3)
    b = O.fill((130,), DType.F32, Dist.NORMAL, 0, 1, 0, 4)
    bv = np.broadcast_to(b, a.shape)
    for op, fn in ((Op.ADD, np.add), (Op.SUB, np.subtract), (Op.MUL, np.multiply), (Op.DIV, np.divide),
                   (Op.MAX, np.maximum), (Op.MIN, np.minimum)):
        out = np.zeros_like(a)
        assert O.eltwise(out, [a, bv], [instr(op, b=1)], Compute.F32) == 0
        assert np.array_equal(out, fn(a, bv)), op.name
    out = np.zeros(a.shape, np.bool_)
    assert O.eltwise(out, [a, bv], [instr(Op.GT, b=1)]) == 0
    assert np.array_equal(out, a > bv)


def test_config2_loop_matches_chain():
    from tadma_b200.abi import DType as D
    x = O.fill((16, 256), D.BF16, Dist.NORMAL, 0, 1, 0, 1)
    bias = O.fill((256,), D.BF16, Dist.NORMAL, 0, 0.1, 0, 2)
    y1 = np.zeros_like(x)
    O.lib().or_cfg2_gelu_affine_bf16(O.ptr(x), O.ptr(bias), 0.5, O.ptr(y1), 16, 256)
    y2 = np.zeros_like(x)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=D.F32), instr(Op.ADD, b=1, round_dtype=D.F32),
            instr(Op.GELU, round_dtype=D.F32)]
    assert O.eltwise(y2, [x, np.broadcast_to(bias, x.shape)], prog, Compute.F32, out_dtype=D.BF16,
                     in_dtypes=[D.BF16, D.BF16]) == 0
    assert np.array_equal(y1, y2)
    xf = bf16_bits_to_f32(x).astype(np.float64) * 0.5 + bf16_bits_to_f32(bias)
    u = 0.7978845608 * (xf + 0.044715 * xf ** 3)
    ref = f32_to_bf16_bits((xf / (1 + np.exp(-2 * u))).astype(np.float32))
    assert np.mean(ref == y1) > 0.99


def test_reduction_kats():
    for n, s in KATS["sum_arange"]:
        x = np.arange(n, dtype=np.int64)[None, :]
        out = np.zeros((1,), np.int64)
        assert O.reduce(Reduce.SUM, x, -1, out) == 0 and out[0] == s
        xf = np.arange(n, dtype=np.float64)[None, :]
        outf = np.zeros((1,), np.float64)
        assert O.reduce(Reduce.MEAN, xf, -1, outf) == 0 and outf[0] == (n - 1) / 2
    rng = np.random.default_rng(1)
    for _ in range(5):
        p = rng.permutation(1000).astype(np.float32)[None, :]
        o = np.zeros((1,), np.int64)
        O.reduce(Reduce.ARGMAX, p, -1, o)
        assert o[0] == int(np.argmax(p))
        O.reduce(Reduce.ARGMIN, p, -1, o)
        assert o[0] == int(np.argmin(p))
    x = np.array([[1.0, 5.0, 5.0, np.nan, 7.0, np.nan]], np.float32)
    o = np.zeros((1,), np.int64)
    O.reduce(Reduce.ARGMAX, x, -1, o)
    assert o[0] == np.argmax(x)  # first NaN, numpy semantics


def test_softmax_and_layer_norm_kats():
    for n, v in KATS["softmax_const_row"]:
        x = np.full((2, n), 3.25, np.float64)
        out = np.zeros_like(x)
        assert O.softmax(x, -1, out) == 0
        np.testing.assert_allclose(out, v, rtol=1e-15)
    row = np.array([KATS["layer_norm_pm1"]["row"]] * 3, np.float64)
    out = np.zeros_like(row)
    for mode in (LNMode.ONNX, LNMode.TADMA):
        assert O.layer_norm(row, -1, None, None, 0.0, mode, out) == 0
        np.testing.assert_allclose(out, np.array([KATS["layer_norm_pm1"]["out"]] * 3), rtol=1e-15)


def test_gather_kats():
    t = np.arange(20, dtype=np.float32).reshape(5, 4)
    ids = np.array([[4, -1], [0, 2]], np.int64)
    out = np.zeros((2, 2, 4), np.float32)
    assert O.gather(t, 0, ids, out) == 0
    assert np.array_equal(out, t[ids % 5])
    out = np.zeros((5, 2, 2), np.float32)
    assert O.gather(t, 1, np.array([[3, 0], [1, 1]], np.int64), out) == 0
    assert np.array_equal(out, t[:, [[3, 0], [1, 1]]])
    bad = np.zeros((1, 4), np.float32)
    assert O.gather(t, 0, np.array([5], np.int64), bad) == 4 and np.all(bad == 0)
