"""The oracle's reference-order reduction against the reference's
ReduceKernel restated on the GPU (baseline/refalgo/refalgo.cu): the same
fold order and accumulator type give the same bits, fp32 and fp16 (fp16
accumulated in fp16).  The library's own reductions accumulate in fp32 in
another order; they are within the stated fp32 tolerance of the exact sum,
which the fp16 reference order is not."""
import ctypes
import os
import subprocess

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tadma_b200.abi import DType, Reduce
import tadma_b200 as tb

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFALGO = os.path.join(ROOT, "baseline", "refalgo", "librefalgo.so")


def refalgo():
    if not os.path.exists(REFALGO):
        subprocess.run(["make", "-s", "-C", os.path.dirname(REFALGO)], check=True)
    L = ctypes.CDLL(REFALGO)
    vp = ctypes.c_void_p
    L.ref_reduce_rows.argtypes = [vp, ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, vp]
    L.ref_reduce_rows.restype = ctypes.c_int
    return L


@pytest.mark.parametrize("dtype", [DType.F32, DType.F16])
@pytest.mark.parametrize("R", [1, 3, 100, 128, 1000, 2048, 4096, 5000])
@pytest.mark.parametrize("op", [0, 1, 2])
def test_restated_reduce_kernel_matches_oracle_bits(dtype, R, op):
    if op == 2 and dtype == DType.F16 and R & (R - 1):
        pytest.skip("fp16 mean: the device's fp16 division is checked at power-of-two R only")
    rows = 64
    rng = np.random.default_rng(R * 7 + op)
    npdt = np.float32 if dtype == DType.F32 else np.float16
    x = (rng.standard_normal((rows, R)) * 4).astype(npdt)
    if op == 1:
        x[3, R // 2] = np.nan  # position-dependent NaN under std::max
    want = O.reduce_rows_reference_order(op, x, dtype)
    tdt = torch.float32 if dtype == DType.F32 else torch.float16
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(rows, dtype=tdt, device="cuda")
    L = refalgo()
    s = torch.cuda.current_stream()
    rc = L.ref_reduce_rows(xd.data_ptr(), 0 if dtype == DType.F32 else 1, out.data_ptr(), rows, R, op, s.cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32 if dtype == DType.F32 else np.uint16),
                          want.view(np.uint32 if dtype == DType.F32 else np.uint16)), (got[:4], want[:4])


def test_library_sum_vs_reference_order_fp16():
    # fp16 rows of 4096 values near 1: fp16 accumulation (the reference)
    # loses the low bits once partials pass 2048; the library accumulates in
    # fp32 and stays within half an fp16 ulp of the exact sum.
    rows, R = 64, 4096
    rng = np.random.default_rng(5)
    x = (1.0 + 0.01 * rng.standard_normal((rows, R))).astype(np.float16)
    exact = x.astype(np.float64).sum(axis=1)
    ref = O.reduce_rows_reference_order(0, x, DType.F16).astype(np.float64)
    out = torch.zeros(rows, dtype=torch.float16, device="cuda")
    tb.reduce(Reduce.SUM, torch.from_numpy(x).cuda(), -1, out)
    torch.cuda.synchronize()
    ours = out.cpu().numpy().astype(np.float64)
    half_ulp = np.spacing(np.abs(exact).astype(np.float16)).astype(np.float64) / 2
    assert np.all(np.abs(ours - exact) <= half_ulp + 1e-2)  # fp32 partial sums, then one rounding
    assert np.abs(ref - exact).max() > np.abs(ours - exact).max()
