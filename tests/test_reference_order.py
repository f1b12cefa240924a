"""The oracle's reference-order reduction (ReduceKernel's fold order and
accumulator type, include/tadma/kernels/Reduce.hpp:10-69) on hand-worked
vectors where the order decides the result (CPU only)."""
import numpy as np

from oracle import oracle as O
from tadma_b200.abi import DType


def test_tree_order_fp32():
    # R = 4: Threads = 4, one element per thread, tree (0 + 2) + (1 + 3):
    # (1e8 + -1e8) + (1 + 1) = 2, where a left-to-right fold gives 1.
    x = np.array([[1e8, 1.0, -1e8, 1.0]], dtype=np.float32)
    assert O.reduce_rows_reference_order(0, x, DType.F32)[0] == np.float32(2.0)
    left_to_right = np.float32(0)
    for v in x[0]:
        left_to_right = np.float32(left_to_right + v)
    assert left_to_right == np.float32(1.0)


def test_strided_fold_fp32():
    # R = 6: Threads = 4; threads 0 and 1 fold elements 4 and 5 first:
    # p = [a0 + a4, a1 + a5, a2, a3], then (p0 + p2) + (p1 + p3).
    a = np.array([[3.0, 1e-8, 5.0, 7.0, 1e8, 1.0]], dtype=np.float32)
    f = np.float32
    p0, p1, p2, p3 = f(a[0, 0] + a[0, 4]), f(a[0, 1] + a[0, 5]), a[0, 2], a[0, 3]
    want = f(f(p0 + p2) + f(p1 + p3))
    assert O.reduce_rows_reference_order(0, a, DType.F32)[0] == want


def test_fp16_accumulates_in_fp16():
    # R = 3: Threads = 2; thread 0 folds 2048 + 1 -> 2048 (fp16 spacing 2,
    # tie to even), then + 1 -> 2048 again; an fp32 accumulator gives 2050.
    x = np.array([[2048, 1, 1]], dtype=np.float16)
    assert O.reduce_rows_reference_order(0, x, DType.F16)[0] == np.float16(2048)
    # mean over R = 4 in fp16: (2048 + 2) + (1 + 1) = 2052 -> / 4 = 513
    y = np.array([[2048, 1, 2, 1]], dtype=np.float16)
    assert O.reduce_rows_reference_order(2, y, DType.F16)[0] == np.float16(513)


def test_max_nan_depends_on_position():
    # std::max(a, b) = a < b ? b : a keeps a NaN only where it is the left
    # operand: tree max(max(1, 3), max(nan, 2)) = max(3, nan) = 3, but
    # max(max(nan, 2), max(1, 3)) = nan.
    x = np.array([[1.0, np.nan, 3.0, 2.0], [np.nan, 1.0, 2.0, 3.0]], dtype=np.float32)
    got = O.reduce_rows_reference_order(1, x, DType.F32)
    assert got[0] == np.float32(3.0) and np.isnan(got[1])
