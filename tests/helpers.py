"""Shared test helpers: host<->device moves, ulp distances, oracle input generation."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O
from tadma_b200.abi import DType, Dist, bf16_bits_to_f32, np_dtype

SEED = 0


def to_dev(a: np.ndarray, dt: DType | None = None):
    """numpy -> torch CUDA tensor (bf16 arrives as raw uint16)."""
    import torch
    a = np.ascontiguousarray(a)
    if dt == DType.BF16 or (dt is None and a.dtype == np.uint16):
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    if a.dtype == np.bool_:
        return torch.from_numpy(a).cuda()
    return torch.from_numpy(a).cuda()


def from_dev(t) -> np.ndarray:
    import torch
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def empty_dev(shape, dt: DType):
    import torch
    tdt = {DType.F32: torch.float32, DType.F16: torch.float16, DType.BF16: torch.bfloat16,
           DType.F64: torch.float64, DType.I64: torch.int64, DType.I32: torch.int32,
           DType.U8: torch.uint8, DType.BOOL: torch.bool, DType.I8: torch.int8}[DType(dt)]
    return torch.full(tuple(shape), 0, dtype=tdt, device="cuda")


def gen(shape, dt: DType, dist: Dist, p0, p1, stream_id, seed=SEED, offset=0) -> np.ndarray:
    return O.fill(tuple(shape), dt, dist, p0, p1, seed, stream_id, offset)


def as_f64(a: np.ndarray, dt: DType) -> np.ndarray:
    if dt == DType.BF16:
        return bf16_bits_to_f32(a).astype(np.float64)
    return a.astype(np.float64)


def ulp_diff(a: np.ndarray, b: np.ndarray, dt: DType) -> np.ndarray:
    """|a - b| in units in the last place of dtype dt (NaN==NaN counts 0)."""
    dt = DType(dt)
    if dt == DType.F32:
        ia, ib = a.astype(np.float32).view(np.int32).astype(np.int64), b.astype(np.float32).view(np.int32).astype(np.int64)
        fa, fb = a.astype(np.float32), b.astype(np.float32)
        lo = -(1 << 31)
    elif dt == DType.F16:
        ia, ib = a.view(np.int16).astype(np.int64), b.view(np.int16).astype(np.int64)
        fa, fb = a.astype(np.float32), b.astype(np.float32)
        lo = -(1 << 15)
    elif dt == DType.BF16:
        ia, ib = a.view(np.int16).astype(np.int64), b.view(np.int16).astype(np.int64)
        fa, fb = bf16_bits_to_f32(a), bf16_bits_to_f32(b)
        lo = -(1 << 15)
    elif dt == DType.F64:
        ia, ib = a.view(np.int64), b.view(np.int64)
        fa, fb = a, b
        lo = None
    else:
        return np.abs(a.astype(np.int64) - b.astype(np.int64))
    if lo is not None:
        ia = np.where(ia < 0, lo - ia, ia)
        ib = np.where(ib < 0, lo - ib, ib)
        d = np.abs(ia - ib)
    else:
        ia = ia.astype(object)
        d = np.abs(np.where(a < 0, -a, a) - np.where(b < 0, -b, b))  # f64 rarely used; coarse
        return d
    both_nan = np.isnan(fa) & np.isnan(fb)
    one_nan = np.isnan(fa) ^ np.isnan(fb)
    d = np.where(both_nan, 0, d)
    d = np.where(one_nan, 1 << 40, d)
    return d


def dev_view(a: np.ndarray, dt: DType):
    """Upload numpy view `a` keeping its broadcast (stride-0) dims as stride 0.

    Returns (keepalive torch tensor, TadmaTensor descriptor with a's shape)."""
    from tadma_b200.abi import make_tensor
    sl = tuple(slice(0, 1) if (s == 0 and n > 1) else slice(None) for s, n in zip(a.strides, a.shape))
    compact = np.ascontiguousarray(a[sl])
    t = to_dev(compact, dt)
    strides = [0 if (s == 0 and n > 1) else ts for s, n, ts in zip(a.strides, a.shape, t.stride())]
    return t, make_tensor(t.data_ptr() if t.numel() else None, dt, list(a.shape), strides)
