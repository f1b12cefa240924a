"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py, never by the product.
PARITY UNPINNED: the oracle restates the reference (which cannot be built
here and has no golden vectors); it is pinned by the analytic KATs in
tests/golden/.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from tadma_b200.abi import (Compute, DType, Op, TadmaInstr, TadmaTensor, host_tensor, program)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    T = TadmaTensor
    c_int, c_double, c_i64, c_u64 = ctypes.c_int32, ctypes.c_double, ctypes.c_int64, ctypes.c_uint64
    vp = ctypes.c_void_p
    L.or_eltwise.argtypes = [P(T), P(T), c_int, P(TadmaInstr), c_int, c_int]
    L.or_reduce.argtypes = [c_int, P(T), c_int, c_int, P(T)]
    L.or_softmax.argtypes = [P(T), c_int, P(T)]
    L.or_layer_norm.argtypes = [P(T), c_int, P(T), P(T), c_double, c_int, P(T)]
    L.or_rms_norm.argtypes = [P(T), c_int, c_double, P(T)]
    L.or_gather.argtypes = [P(T), c_int, P(T), P(T), P(T)]
    L.or_fill.argtypes = [P(T), c_int, c_double, c_double, c_u64, c_u64, c_i64]
    L.or_map_to_shape.argtypes = [P(c_i64), c_int, c_i64, P(c_i64)]
    L.or_mix64.argtypes = [c_u64]
    L.or_mix64.restype = c_u64
    L.or_f32_to_f16.argtypes = [ctypes.c_float]
    L.or_f32_to_f16.restype = ctypes.c_uint16
    L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.or_f16_to_f32.restype = ctypes.c_float
    L.or_f32_to_bf16.argtypes = [ctypes.c_float]
    L.or_f32_to_bf16.restype = ctypes.c_uint16
    L.or_bf16_to_f32.argtypes = [ctypes.c_uint16]
    L.or_bf16_to_f32.restype = ctypes.c_float
    L.or_cfg2_gelu_affine_bf16.argtypes = [vp, vp, ctypes.c_float, vp, c_i64, c_i64]
    L.or_cfg3_sum_lastaxis_f32.argtypes = [vp, vp, c_i64, c_i64]
    L.or_cfg3_max_lastaxis_f32.argtypes = [vp, vp, c_i64, c_i64]
    L.or_cfg3_argmax_lastaxis_f32.argtypes = [vp, vp, c_i64, c_i64]
    L.or_cfg3_mean_midaxis_f32.argtypes = [vp, vp, c_i64, c_i64, c_i64]
    L.or_cfg4_layer_norm_f16.argtypes = [vp, vp, vp, c_double, vp, c_i64, c_i64]
    L.or_cfg4_softmax_f16.argtypes = [vp, vp, c_i64, c_i64]
    L.or_cfg5_gather_add.argtypes = [vp, c_i64, vp, vp, vp, c_i64, c_i64, c_i64]
    L.or_reduce_rows_reference_order.argtypes = [c_int, vp, c_int, c_i64, c_i64, vp]
    L.or_reduce_rows_reference_order.restype = c_int
    L.or_num_threads.restype = c_int
    L.or_set_num_threads.argtypes = [c_int]
    for name in ("or_eltwise", "or_reduce", "or_softmax", "or_layer_norm", "or_rms_norm", "or_gather", "or_fill"):
        getattr(L, name).restype = c_int
    _lib = L
    return L


def _t(a, dt=None):
    return host_tensor(a, dt) if a is not None else TadmaTensor()


def fill(shape, dtype, dist, p0, p1, seed, stream_id, offset=0) -> np.ndarray:
    from tadma_b200.abi import np_dtype
    a = np.zeros(shape, dtype=np_dtype(dtype))
    rc = lib().or_fill(ctypes.byref(host_tensor(a, dtype)), int(dist), float(p0), float(p1), int(seed),
                       int(stream_id), int(offset))
    assert rc == 0, rc
    return a


def eltwise(out: np.ndarray, ins, prog, compute=Compute.AUTO, out_dtype=None, in_dtypes=None) -> int:
    """ins: list of numpy arrays (already broadcast-shaped views allowed via strides)."""
    in_dtypes = in_dtypes or [None] * len(ins)
    arr = (TadmaTensor * max(1, len(ins)))(*[_t(a, d) for a, d in zip(ins, in_dtypes)])
    p, n = program(prog)
    return lib().or_eltwise(ctypes.byref(_t(out, out_dtype)), arr, len(ins), p, n, int(compute))


def reduce(op, x, axis, out, pre_op=Op.COPY, x_dtype=None, out_dtype=None) -> int:
    return lib().or_reduce(int(op), ctypes.byref(_t(x, x_dtype)), int(axis), int(pre_op),
                           ctypes.byref(_t(out, out_dtype)))


def reduce_rows_reference_order(op: int, x: np.ndarray, dtype: int) -> np.ndarray:
    """Row reductions of a 2-D array in the reference's ReduceKernel fold
    order and accumulator type (op 0 sum, 1 max, 2 mean; dtype F32 or F16,
    fp16 given as np.float16)."""
    x = np.ascontiguousarray(x)
    rows, R = x.shape
    out = np.zeros(rows, dtype=x.dtype)
    rc = lib().or_reduce_rows_reference_order(int(op), x.ctypes.data, int(dtype), rows, R, out.ctypes.data)
    if rc != 0:
        raise ValueError("unsupported dtype or op")
    return out


def softmax(x, axis, out, dtype=None) -> int:
    return lib().or_softmax(ctypes.byref(_t(x, dtype)), int(axis), ctypes.byref(_t(out, dtype)))


def layer_norm(x, axis, gamma, beta, eps, mode, out, dtype=None, gb_dtype=None) -> int:
    return lib().or_layer_norm(ctypes.byref(_t(x, dtype)), int(axis), ctypes.byref(_t(gamma, gb_dtype)),
                               ctypes.byref(_t(beta, gb_dtype)), float(eps), int(mode), ctypes.byref(_t(out, dtype)))


def rms_norm(x, axis, eps, out, dtype=None) -> int:
    return lib().or_rms_norm(ctypes.byref(_t(x, dtype)), int(axis), float(eps), ctypes.byref(_t(out, dtype)))


def gather(table, axis, ids, out, add=None, table_dtype=None, add_dtype=None, out_dtype=None) -> int:
    return lib().or_gather(ctypes.byref(_t(table, table_dtype)), int(axis), ctypes.byref(_t(ids)),
                           ctypes.byref(_t(add, add_dtype)), ctypes.byref(_t(out, out_dtype)))


def map_to_shape(dims, index):
    n = len(dims)
    d = (ctypes.c_int64 * n)(*dims)
    o = (ctypes.c_int64 * n)()
    lib().or_map_to_shape(d, n, int(index), o)
    return list(o)


def ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)
