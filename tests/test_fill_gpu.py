"""Device generator (tadma_b200_fill) vs the oracle generator: bit-exact."""
import numpy as np
import pytest

import tadma_b200 as tb
from tadma_b200.abi import DType, Dist, make_tensor
from tests.helpers import empty_dev, from_dev, gen

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", [DType.F32, DType.F16, DType.BF16, DType.F64])
@pytest.mark.parametrize("dist,p0,p1", [(Dist.NORMAL, 0.0, 1.0), (Dist.NORMAL, 1.0, 0.02), (Dist.UNIFORM, -1.0, 1.0),
                                        (Dist.NORMAL, 0.0, 3.0)])
def test_fill_float_bit_exact(dt, dist, p0, p1):
    shape = (37, 1031)
    t = empty_dev(shape, dt)
    tb.fill(t, dist, p0, p1, seed=7, stream_id=11, offset=123)
    ref = gen(shape, dt, dist, p0, p1, stream_id=11, seed=7, offset=123)
    assert np.array_equal(from_dev(t).view(np.uint8), ref.view(np.uint8))


@pytest.mark.parametrize("dt", [DType.I64, DType.I32])
def test_fill_index_bit_exact(dt):
    shape = (64, 257)
    t = empty_dev(shape, dt)
    tb.fill(t, Dist.INDEX, 0, 50257, seed=0, stream_id=5)
    ref = gen(shape, dt, Dist.INDEX, 0, 50257, stream_id=5)
    got = from_dev(t)
    assert np.array_equal(got, ref)
    assert got.min() >= 0 and got.max() < 50257


def test_fill_strided_and_sharded():
    # A transposed view gets element (i, j) of the logical row-major order;
    # a shard at offset k equals rows k.. of the full tensor.
    base = empty_dev((64, 48), DType.F32)
    view = make_tensor(base.data_ptr(), DType.F32, [48, 64], [1, 48])
    tb.fill(view, Dist.NORMAL, 0.0, 1.0, seed=3, stream_id=9)
    ref = gen((48, 64), DType.F32, Dist.NORMAL, 0.0, 1.0, stream_id=9, seed=3)
    assert np.array_equal(from_dev(base).T, ref)
    shard = empty_dev((16, 64), DType.F32)
    tb.fill(shard, Dist.NORMAL, 0.0, 1.0, seed=3, stream_id=9, offset=32 * 64)
    assert np.array_equal(from_dev(shard), ref[32:])
