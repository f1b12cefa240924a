"""Runs tests/cpp/conformance.cu (generated-code-style calls of the header-only
Tensor API) on the GPU and checks every result against the oracle on the same
seeded inputs (regenerated on the host by the oracle's generator)."""
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, LNMode, Op, Reduce, bf16_bits_to_f32, instr
from tests.cpp_build import build_conformance
from tests.helpers import ulp_diff

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    d = tmp_path_factory.mktemp("conf")
    exe = build_conformance(str(d))
    r = subprocess.run([exe, str(d)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "conformance ok" in r.stdout

    def load(name, dtype, shape):
        a = np.fromfile(os.path.join(d, name + ".bin"), dtype=dtype)
        return a.reshape(shape)
    return load


def gen(shape, dt, dist, p0, p1, sid):
    return O.fill(shape, dt, dist, p0, p1, 0, sid)


def test_config2_operators_and_fused(results):
    x = gen((64, 1024), DType.BF16, Dist.NORMAL, 0.0, 1.0, 1)
    bias = gen((1024,), DType.BF16, Dist.NORMAL, 0.0, 0.1, 2)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
            instr(Op.GELU, round_dtype=DType.F32)]
    ref = np.zeros((64, 1024), np.float32)
    O.eltwise(ref, [x, np.broadcast_to(bias, x.shape)], prog, Compute.F32, out_dtype=DType.F32,
              in_dtypes=[DType.BF16, DType.BF16])
    got = results("cfg2_ops_f32", np.float32, (64, 1024))
    assert ulp_diff(got, ref, DType.F32).max() <= 64
    refb = np.zeros((64, 1024), np.uint16)
    O.eltwise(refb, [x, np.broadcast_to(bias, x.shape)], prog, Compute.F32, out_dtype=DType.BF16,
              in_dtypes=[DType.BF16, DType.BF16])
    gotb = results("cfg2_fused_bf16", np.uint16, (64, 1024))
    assert ulp_diff(gotb, refb, DType.BF16).max() <= 1


def test_config1(results):
    A = gen((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 1)
    b = gen((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 2)
    e = np.exp((A + b).astype(np.float64))
    got = results("cfg1_sum", np.float32, (64,))
    np.testing.assert_allclose(got, e.sum(axis=1), rtol=1e-5 * np.sqrt(128))
    got = results("cfg1_fused_sum", np.float32, (64,))
    np.testing.assert_allclose(got, e.sum(axis=1), rtol=1e-5 * np.sqrt(128))


def test_config3(results):
    X = gen((2, 64, 256), DType.F32, Dist.UNIFORM, -1.0, 1.0, 3)
    Xd = X.astype(np.float64)
    np.testing.assert_allclose(results("cfg3_sum", np.float32, (2, 64, 1)), Xd.sum(-1, keepdims=True), atol=1e-5 * 16 * 16)
    assert np.array_equal(results("cfg3_max", np.float32, (2, 64, 1)), X.max(-1, keepdims=True))
    assert np.array_equal(results("cfg3_argmax", np.int64, (2, 64)), X.argmax(-1))
    np.testing.assert_allclose(results("cfg3_mean1", np.float32, (2, 1, 256)), Xd.mean(1, keepdims=True), atol=1e-6)


def test_config4(results):
    L = gen((4, 16, 1024), DType.F16, Dist.NORMAL, 0.0, 1.0, 4)
    g = gen((1024,), DType.F16, Dist.NORMAL, 1.0, 0.02, 5)
    be = gen((1024,), DType.F16, Dist.NORMAL, 0.0, 0.02, 6)
    for name, mode in (("cfg4_ln", LNMode.ONNX), ("cfg4_ln_tadma", LNMode.TADMA)):
        ref = np.zeros_like(L)
        O.layer_norm(L, -1, g, be, 1e-5, mode, ref)
        assert ulp_diff(results(name, np.float16, L.shape), ref, DType.F16).max() <= 1, name
    S = gen((2, 4, 256, 2048), DType.F16, Dist.NORMAL, 0.0, 3.0, 7)
    ref = np.zeros_like(S)
    O.softmax(S, -1, ref)
    assert ulp_diff(results("cfg4_softmax", np.float16, S.shape), ref, DType.F16).max() <= 1


def test_config5(results):
    table = gen((1000, 256), DType.F16, Dist.NORMAL, 0.0, 0.02, 8)
    ids = gen((4, 64), DType.I64, Dist.INDEX, 0, 1000, 9)
    pos = gen((64, 256), DType.BF16, Dist.NORMAL, 0.0, 0.02, 10)
    want = table[ids].astype(np.float32) + bf16_bits_to_f32(pos)[None]
    assert np.array_equal(results("cfg5_gather_add_f32", np.float32, (4, 64, 256)), want)
    assert np.array_equal(results("cfg5_gather", np.float16, (4, 64, 256)), table[ids])


def test_generated_layer_norm_chain(results):
    h = gen((2, 8, 768), DType.F32, Dist.NORMAL, 0.0, 1.0, 11).astype(np.float64)
    w = gen((768,), DType.F32, Dist.NORMAL, 1.0, 0.02, 12).astype(np.float64)
    wb = gen((768,), DType.F32, Dist.NORMAL, 0.0, 0.02, 13).astype(np.float64)
    m = h.mean(-1, keepdims=True)
    v = ((h - m) ** 2).mean(-1, keepdims=True)
    ref = (h - m) / np.sqrt(v + 9.999999960041972e-13) * w + wb
    got = results("gen_ln", np.float64, (2, 8, 768))  # var + a double constant promotes to double
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_views_and_copies(results):
    X = gen((2, 64, 256), DType.F32, Dist.UNIFORM, -1.0, 1.0, 3)
    assert np.array_equal(results("view_transpose", np.float32, (2, 256, 64)), X.transpose(0, 2, 1))
    assert np.array_equal(results("view_slice", np.float32, (2, 4, 256)), X[:, 1:9:2])
    np.testing.assert_allclose(results("view_reshape_sum", np.float32, (2,)), X.reshape(2, -1).astype(np.float64).sum(1),
                               atol=1e-2)
    assert np.array_equal(results("concat", np.float32, (2, 72, 256)), np.concatenate([X, X[:, :8]], axis=1))
    assert np.array_equal(results("where", np.float32, X.shape), np.where(X > 0.25, X, X * np.float32(-1)))
    assert np.array_equal(results("cast_f16", np.float16, X.shape), X.astype(np.float16))
    A = gen((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 1)
    b = gen((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 2)
    assert np.array_equal(results("unsqueeze_bcast_add", np.float32, (64, 128)), A + b[None, :])


def test_generated_shape_arithmetic(results):
    # GraphPrologue in tests/cpp/conformance.cu: position ids sliced from a
    # ConstexprAllocator constant by a shape computed at compile time, word +
    # position embeddings, Reshape by a concatenated shape, Expand by type.
    word = gen((100, 32), DType.F32, Dist.NORMAL, 0.0, 1.0, 14)
    pos = gen((16, 32), DType.F32, Dist.NORMAL, 0.0, 1.0, 15)
    ids = gen((2, 12), DType.I64, Dist.INDEX, 0, 100, 16)
    assert np.array_equal(results("gen_position_ids", np.int64, (12,)), np.arange(12))
    emb = (word[ids] + pos[:12][None]).astype(np.float32)
    assert np.array_equal(results("gen_embed_flat", np.float32, (2, 12 * 32)), emb.reshape(2, -1))
    assert np.array_equal(results("gen_expand", np.float32, (2, 12, 32)), np.broadcast_to(pos[:12], (2, 12, 32)))


# Lazy chains (include/tadma/Lazy.hpp): each lazy result is compared with the
# same calls made eagerly, one kernel per op.  Element-wise chains and
# max / argmin are bit-identical: every step rounds to the eager result type
# and computes in the eager precision.  Sums differ only in their order.
LAZY_PAIRS = [
    ("cfg2", np.float32, (64, 1024)),
    ("cfg2_f64", np.float64, (64, 1024)),
    ("max", np.float32, (2, 64, 1)),
    ("argmin1", np.int64, (2, 256)),
    ("rev", np.float32, (64, 128)),
    ("cmp", np.bool_, (64, 128)),
    ("int", np.float64, (4, 64)),
    ("long", np.float32, (64, 128)),
    ("operands", np.float32, (64, 128)),
    ("square", np.float32, (64, 128)),
    ("where", np.float32, (64, 128)),
    ("softmax", np.float32, (2, 4, 256, 2048)),
    ("softmax_then", np.float32, (2, 4, 256, 1)),
]


@pytest.mark.parametrize("name,dt,shape", LAZY_PAIRS)
def test_lazy_chain_equals_eager_calls(results, name, dt, shape):
    lazy, eager = results("lazy_" + name, dt, shape), results("eager_" + name, dt, shape)
    assert np.array_equal(lazy.view(np.uint8), eager.view(np.uint8)), name


def test_lazy_reductions(results):
    # config 1 through lazy values: exp<false>(lazy(A) + b).sum<-1, false>()
    # is the fused_reduce call (one kernel), bit for bit
    A = gen((64, 128), DType.F32, Dist.NORMAL, 0.0, 1.0, 1)
    b = gen((128,), DType.F32, Dist.NORMAL, 0.0, 1.0, 2)
    got = results("lazy_cfg1_sum", np.float32, (64,))
    assert np.array_equal(got, results("cfg1_fused_sum", np.float32, (64,)))
    np.testing.assert_allclose(got, np.exp((A + b).astype(np.float64)).sum(axis=1), rtol=1e-5 * np.sqrt(128))
    # tanh(lazy(L).to<float>()).sum<-1>() against the eager cast, tanh and row sum
    lazy, eager = results("lazy_cast_sum", np.float32, (4, 16, 1)), results("eager_cast_sum", np.float32, (4, 16, 1))
    L = gen((4, 16, 1024), DType.F16, Dist.NORMAL, 0.0, 1.0, 4).astype(np.float64)
    np.testing.assert_allclose(lazy, eager, rtol=1e-5 * 32, atol=1e-5 * 32)
    np.testing.assert_allclose(lazy, np.tanh(L).sum(-1, keepdims=True), rtol=1e-5 * 32, atol=1e-4)
    # where with a lazy condition, reduced in the same kernel
    X = gen((2, 64, 256), DType.F32, Dist.UNIFORM, -1.0, 1.0, 3).astype(np.float64)
    lazy, eager = results("lazy_where_sum", np.float32, (2, 64, 1)), results("eager_where_sum", np.float32, (2, 64, 1))
    ref = np.where(X < 0, X * 0.5, X).sum(-1, keepdims=True)
    np.testing.assert_allclose(lazy, eager, atol=1e-5 * 16)
    np.testing.assert_allclose(lazy, ref, atol=1e-5 * 16)
