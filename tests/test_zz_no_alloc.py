"""tadma_b200_reduce_noalloc: the reduction entry point for callers that
cannot allocate device memory (a process whose pool already holds the HBM, a
latency-critical path that must not enter the allocator).  Its long-axis
partials live in the library's 2 MiB static device buffer instead of a
per-call workspace.

Called through the C ABI and compared with tadma_b200_reduce on the same
inputs, twice in a row (the second call finds the first call's partials still
in the shared buffer), within the reduction tolerance of tests/test_reduce_gpu.py.
Kept in its own file, collected last, and independent of the other tests.
"""
import ctypes

import numpy as np
import pytest

import tadma_b200 as tb
from tadma_b200.abi import Dist, DType, Reduce

pytestmark = pytest.mark.gpu


def _reduce(entry, op, x, axis, out):
    import torch
    i, o = tb.desc(x), tb.desc(out)
    rc = entry(int(op), ctypes.byref(i), int(axis), 0, ctypes.byref(o),
               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return rc


def _close(a, b, n, exact=False):
    a, b = a.double().cpu().numpy(), b.double().cpu().numpy()
    if exact:
        return np.array_equal(a, b)
    return np.all(np.abs(a - b) <= 1e-5 * np.sqrt(n) * np.maximum(np.abs(b), 1.0))


@pytest.mark.parametrize("shape,axis,op,dt", [
    ((3, 200003), -1, Reduce.SUM, DType.F32),      # long rows: split across CTAs
    ((2, 1 << 21), -1, Reduce.ARGMAX, DType.BF16),
    ((2, 100000, 64), 1, Reduce.MEAN, DType.F32),  # long strided axis: column split
    ((4, 4096, 33), 1, Reduce.MAX, DType.F16),
    ((64, 128), -1, Reduce.SUM, DType.F32),        # no split: needs no scratch at all
])
def test_noalloc_matches_reduce_twice(shape, axis, op, dt):
    import torch
    L = tb.lib()
    tdt = {DType.F32: torch.float32, DType.BF16: torch.bfloat16, DType.F16: torch.float16}[dt]
    x = torch.empty(shape, dtype=tdt, device="cuda")
    oshape = list(shape)
    oshape[axis] = 1
    odt = torch.int64 if op == Reduce.ARGMAX else torch.float32
    n = shape[axis]
    for call in range(2):
        tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=call, stream_id=40)
        want = torch.empty(oshape, dtype=odt, device="cuda")
        got = torch.full(oshape, -7, dtype=odt, device="cuda")
        assert _reduce(L.tadma_b200_reduce, op, x, axis, want) == 0
        assert _reduce(L.tadma_b200_reduce_noalloc, op, x, axis, got) == 0, L.tadma_b200_last_error()
        assert _close(got, want, n, exact=op == Reduce.ARGMAX), (call, shape)


@pytest.mark.parametrize("shape", [
    (1, 4096, 36864),  # 144 column tiles; a wave of CTAs needs 6 partial slots of 36864 x 16 bytes: 3 fit
    (1, 4096, 70000),  # one split's partials (1.1 MB) leave no room for two: one pass, no scratch
])
def test_noalloc_fits_its_split_to_the_static_scratch(shape):
    import torch
    L = tb.lib()
    x = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=3, stream_id=41)
    oshape = (shape[0], 1, shape[2])
    want = torch.empty(oshape, dtype=torch.float32, device="cuda")
    got = torch.full(oshape, -7.0, dtype=torch.float32, device="cuda")
    assert _reduce(L.tadma_b200_reduce, Reduce.SUM, x, 1, want) == 0
    for _ in range(2):
        assert _reduce(L.tadma_b200_reduce_noalloc, Reduce.SUM, x, 1, got) == 0, L.tadma_b200_last_error()
        assert _close(got, want, shape[1])


def test_noalloc_on_two_devices():
    """The static buffer's address is looked up per device: a call on cuda:1
    after one on cuda:0 must use cuda:1's copy of the buffer."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    L = tb.lib()
    for dev in (0, 1, 0, 1):
        with torch.cuda.device(dev):
            x = torch.empty((3, 200003), dtype=torch.float32, device="cuda")
            tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=dev, stream_id=42)
            want = torch.empty((3, 1), dtype=torch.float32, device="cuda")
            got = torch.full((3, 1), -7.0, dtype=torch.float32, device="cuda")
            assert _reduce(L.tadma_b200_reduce, Reduce.SUM, x, -1, want) == 0
            assert _reduce(L.tadma_b200_reduce_noalloc, Reduce.SUM, x, -1, got) == 0, L.tadma_b200_last_error()
            assert _close(got, want, 200003)
