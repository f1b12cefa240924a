"""tadma_b200: B200 (sm_100a) kernels behind TADMA's Tensor API, Python binding.

The product is the C-ABI library ``libtadma_b200.so`` built in-tree from
``tadma_b200/csrc`` (declared in ``include/tadma_b200.h``).  This module loads
it with ctypes and offers thin helpers that build descriptors from torch CUDA
tensors.  torch is used for device memory and streams only; every op runs the
library's own kernels.  There is no CPU fallback: if the library is missing the
import raises.
"""
from __future__ import annotations

import ctypes
import os

from .abi import (  # noqa: F401  (re-exported)
    MAX_INPUTS, MAX_INSTR, MAX_RANK, ROWPROG_MAX_STAGES, SRC_IMM, SRC_NONE, BINARY_OPS, TRANSCENDENTAL, UNARY_OPS,
    Compute, Dist, DType, LNMode, Op, Reduce, Status, TadmaInstr, TadmaRowProgram, TadmaRowStage, TadmaTensor,
    instr, make_tensor, program,
)

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtadma_b200.so")

_lib = None

EXPORTS = (
    "tadma_b200_eltwise", "tadma_b200_reduce", "tadma_b200_softmax", "tadma_b200_layer_norm",
    "tadma_b200_rms_norm", "tadma_b200_gather", "tadma_b200_fill", "tadma_b200_last_error",
    "tadma_b200_version", "tadma_b200_error_flags", "tadma_b200_dtype_size", "tadma_b200_reduce_noalloc",
    "tadma_b200_reduce_chain", "tadma_b200_reduce_chain_post", "tadma_b200_row_program",
)


class TadmaError(RuntimeError):
    """A C-ABI call returned a non-zero status (code + the library's message)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{Status(code).name}: {msg}")
        self.code = code


def lib() -> ctypes.CDLL:
    """Load libtadma_b200.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    T, I = TadmaTensor, TadmaInstr
    c_int, c_void, c_double = ctypes.c_int32, ctypes.c_void_p, ctypes.c_double
    L.tadma_b200_eltwise.argtypes = [P(T), P(T), c_int, P(I), c_int, c_int, c_void]
    L.tadma_b200_reduce.argtypes = [c_int, P(T), c_int, c_int, P(T), c_void]
    L.tadma_b200_reduce_noalloc.argtypes = [c_int, P(T), c_int, c_int, P(T), c_void]
    L.tadma_b200_reduce_chain.argtypes = [c_int, P(T), c_int, P(I), c_int, c_int, c_int, P(T), c_void]
    L.tadma_b200_reduce_chain_post.argtypes = [c_int, P(T), c_int, P(I), c_int, P(I), c_int, c_int, c_int, P(T),
                                               c_void]
    L.tadma_b200_row_program.argtypes = [P(TadmaRowProgram), c_void]
    L.tadma_b200_softmax.argtypes = [P(T), c_int, P(T), c_void]
    L.tadma_b200_layer_norm.argtypes = [P(T), c_int, P(T), P(T), c_double, c_int, P(T), c_void]
    L.tadma_b200_rms_norm.argtypes = [P(T), c_int, c_double, P(T), c_void]
    L.tadma_b200_gather.argtypes = [P(T), c_int, P(T), P(T), P(T), c_void]
    L.tadma_b200_fill.argtypes = [P(T), c_int, c_double, c_double, ctypes.c_uint64, ctypes.c_uint64,
                                  ctypes.c_int64, c_void]
    L.tadma_b200_error_flags.argtypes = [P(ctypes.c_uint32), c_int]
    L.tadma_b200_dtype_size.argtypes = [c_int]
    for name in EXPORTS:
        getattr(L, name).restype = ctypes.c_int32
    L.tadma_b200_last_error.restype = ctypes.c_char_p
    L.tadma_b200_version.restype = ctypes.c_char_p
    L.tadma_b200_last_error.argtypes = []
    L.tadma_b200_version.argtypes = []
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != 0:
        raise TadmaError(rc, lib().tadma_b200_last_error().decode())


def version() -> str:
    return lib().tadma_b200_version().decode()


# ---------------------------------------------------------------- torch glue --

def _torch():
    import torch
    return torch


_TORCH_DT = None


def torch_dtype_code(t) -> DType:
    global _TORCH_DT
    torch = _torch()
    if _TORCH_DT is None:
        _TORCH_DT = {torch.float32: DType.F32, torch.float16: DType.F16, torch.bfloat16: DType.BF16,
                     torch.float64: DType.F64, torch.int64: DType.I64, torch.int32: DType.I32,
                     torch.uint8: DType.U8, torch.bool: DType.BOOL, torch.int8: DType.I8}
    return _TORCH_DT[t.dtype]


def desc(t, shape=None, strides=None) -> TadmaTensor:
    """Descriptor of a torch tensor (optionally re-viewed with shape/strides in elements)."""
    return make_tensor(t.data_ptr() if t.numel() else None, torch_dtype_code(t),
                       list(t.shape) if shape is None else shape,
                       list(t.stride()) if strides is None else strides)


def none_tensor() -> TadmaTensor:
    return TadmaTensor()


def _stream(stream):
    if stream is None:
        return ctypes.c_void_p(_torch().cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


class Prepared:
    """A C-ABI call with its ctypes arguments built once (descriptors, program,
    stream): calling it costs one foreign call, for launch-bound loops.  The
    stream is fixed when the call is prepared (the current torch stream when
    none is given); prepare on the capture stream to record into a CUDA graph."""

    def __init__(self, fn, args, keep=()):
        self._fn, self._args, self._keep = fn, args, keep

    def __call__(self) -> None:
        rc = self._fn(*self._args)
        if rc != 0:
            check(rc)


def _d(t):
    return t if isinstance(t, TadmaTensor) else desc(t)


def prepare_eltwise(out, ins, prog, compute=Compute.AUTO, stream=None) -> Prepared:
    o = _d(out)
    arr = (TadmaTensor * max(1, len(ins)))(*[_d(x) for x in ins])
    p, n = program(prog)
    return Prepared(lib().tadma_b200_eltwise, (ctypes.byref(o), arr, len(ins), p, n, int(compute), _stream(stream)),
                    (o, arr, p))


def prepare_reduce(op, x, axis, out, pre_op=Op.COPY, stream=None) -> Prepared:
    i, o = _d(x), _d(out)
    return Prepared(lib().tadma_b200_reduce, (int(op), ctypes.byref(i), int(axis), int(pre_op), ctypes.byref(o),
                                              _stream(stream)), (i, o))


def prepare_reduce_chain(op, ins, prog, axis, out, compute=Compute.AUTO, stream=None, post=None) -> Prepared:
    """out = reduce `op` over `axis` of chain(ins...) in one kernel (tadma_b200_reduce_chain); with `post`
    (instructions with immediate operands), out = post(reduce(...)) (tadma_b200_reduce_chain_post)."""
    arr = (TadmaTensor * max(1, len(ins)))(*[_d(x) for x in ins])
    p, n = program(prog)
    o = _d(out)
    if post:
        q, m = program(post)
        return Prepared(lib().tadma_b200_reduce_chain_post, (int(op), arr, len(ins), p, n, q, m, int(compute),
                                                             int(axis), ctypes.byref(o), _stream(stream)),
                        (arr, p, q, o))
    return Prepared(lib().tadma_b200_reduce_chain, (int(op), arr, len(ins), p, n, int(compute), int(axis),
                                                    ctypes.byref(o), _stream(stream)), (arr, p, o))


def prepare_softmax(x, axis, out, stream=None) -> Prepared:
    i, o = _d(x), _d(out)
    return Prepared(lib().tadma_b200_softmax, (ctypes.byref(i), int(axis), ctypes.byref(o), _stream(stream)), (i, o))


def prepare_layer_norm(x, axis, gamma, beta, eps, out, mode=LNMode.ONNX, stream=None) -> Prepared:
    i, o = _d(x), _d(out)
    g = none_tensor() if gamma is None else _d(gamma)
    b = none_tensor() if beta is None else _d(beta)
    return Prepared(lib().tadma_b200_layer_norm, (ctypes.byref(i), int(axis), ctypes.byref(g), ctypes.byref(b),
                                                  float(eps), int(mode), ctypes.byref(o), _stream(stream)), (i, o, g, b))


def prepare_rms_norm(x, axis, eps, out, stream=None) -> Prepared:
    i, o = _d(x), _d(out)
    return Prepared(lib().tadma_b200_rms_norm, (ctypes.byref(i), int(axis), float(eps), ctypes.byref(o),
                                                _stream(stream)), (i, o))


def prepare_gather(table, axis, ids, out, add=None, stream=None) -> Prepared:
    t, i, o = _d(table), _d(ids), _d(out)
    a = none_tensor() if add is None else _d(add)
    return Prepared(lib().tadma_b200_gather, (ctypes.byref(t), int(axis), ctypes.byref(i), ctypes.byref(a),
                                              ctypes.byref(o), _stream(stream)), (t, i, o, a))


def prepare_fill(out, dist, p0, p1, seed, stream_id, offset=0, stream=None) -> Prepared:
    o = _d(out)
    return Prepared(lib().tadma_b200_fill, (ctypes.byref(o), int(dist), float(p0), float(p1), int(seed),
                                            int(stream_id), int(offset), _stream(stream)), (o,))


def eltwise(out, ins, prog, compute=Compute.AUTO, stream=None) -> None:
    """out = chain(ins...) (tadma_b200_eltwise).  `out`/`ins` are torch tensors or descriptors."""
    prepare_eltwise(out, ins, prog, compute, stream)()


def reduce(op, x, axis, out, pre_op=Op.COPY, stream=None) -> None:
    prepare_reduce(op, x, axis, out, pre_op, stream)()


def reduce_chain(op, ins, prog, axis, out, compute=Compute.AUTO, stream=None, post=None) -> None:
    prepare_reduce_chain(op, ins, prog, axis, out, compute, stream, post)()


def row_program(rows, cols, ins, stages, prog, out, acc=0, compute=Compute.F32, stream=None) -> None:
    """tadma_b200_row_program.  ins: descriptors (or torch tensors) viewed as
    {rows, cols}; stages: (op, chain, post, out, acc) tuples, out a {rows}
    descriptor or tensor; prog: the final chain; out: {rows, cols}."""
    rp = TadmaRowProgram()
    rp.rows, rp.cols = int(rows), int(cols)
    rp.n_ins = len(ins)
    for k, t in enumerate(ins):
        rp.ins[k] = _d(t)
    rp.n_stages = len(stages)
    for s, (op, chain, post, sout, sacc) in enumerate(stages):
        st = rp.stages[s]
        st.op, st.n_instr, st.n_post, st.acc = int(op), len(chain), len(post), int(sacc)
        for i, I in enumerate(chain):
            st.prog[i] = I
        for i, I in enumerate(post):
            st.post[i] = I
        st.out = _d(sout)
    rp.n_instr = len(prog)
    for i, I in enumerate(prog):
        rp.prog[i] = I
    rp.acc = int(acc)
    rp.compute = int(compute)
    rp.out = _d(out)
    check(lib().tadma_b200_row_program(ctypes.byref(rp), _stream(stream)))


def softmax(x, axis, out, stream=None) -> None:
    prepare_softmax(x, axis, out, stream)()


def layer_norm(x, axis, gamma, beta, eps, out, mode=LNMode.ONNX, stream=None) -> None:
    prepare_layer_norm(x, axis, gamma, beta, eps, out, mode, stream)()


def rms_norm(x, axis, eps, out, stream=None) -> None:
    prepare_rms_norm(x, axis, eps, out, stream)()


def gather(table, axis, ids, out, add=None, stream=None) -> None:
    prepare_gather(table, axis, ids, out, add, stream)()


def fill(out, dist, p0, p1, seed, stream_id, offset=0, stream=None) -> None:
    prepare_fill(out, dist, p0, p1, seed, stream_id, offset, stream)()


def error_flags(clear: bool = True) -> int:
    w = ctypes.c_uint32(0)
    check(lib().tadma_b200_error_flags(ctypes.byref(w), 1 if clear else 0))
    return int(w.value)
