"""ctypes mirror of include/tadma_b200.h: structs, enums and descriptor helpers.

Pure ABI definitions; importing this module loads no library.  Both the CUDA
library binding (tadma_b200/__init__.py) and the host oracle binding share it,
and tests/test_abi.py checks every constant here against the C header.
"""
from __future__ import annotations

import ctypes
import enum

import numpy as np

MAX_RANK = 8
MAX_INPUTS = 6
MAX_INSTR = 16
SRC_IMM = -1
SRC_NONE = -2


class DType(enum.IntEnum):
    F32 = 0
    F16 = 1
    BF16 = 2
    F64 = 3
    I64 = 4
    I32 = 5
    U8 = 6
    BOOL = 7
    I8 = 8


class Status(enum.IntEnum):
    OK = 0
    ERR_INVALID = 1
    ERR_UNSUPPORTED = 2
    ERR_CUDA = 3
    ERR_INDEX = 4


class Op(enum.IntEnum):
    COPY = 0
    NEG = 1
    ABS = 2
    EXP = 3
    LOG = 4
    SQRT = 5
    SIN = 6
    COS = 7
    TAN = 8
    ASIN = 9
    ACOS = 10
    ATAN = 11
    ASINH = 12
    ACOSH = 13
    ATANH = 14
    ERF = 15
    RELU = 16
    SIGMOID = 17
    TANH = 18
    GELU = 19
    NOT = 20
    ADD = 32
    SUB = 33
    MUL = 34
    DIV = 35
    POW = 36
    RSUB = 37
    RDIV = 38
    MAX = 39
    MIN = 40
    EQ = 41
    NE = 42
    LT = 43
    GT = 44
    LE = 45
    GE = 46
    AND = 47
    OR = 48
    XOR = 49
    LAND = 50
    LOR = 51
    WHERE = 64


class Compute(enum.IntEnum):
    AUTO = -1
    F32 = 0
    F64 = 1
    I64 = 2
    F32_PRECISE = 3


class Reduce(enum.IntEnum):
    SUM = 0
    MEAN = 1
    MAX = 2
    MIN = 3
    ARGMAX = 4
    ARGMIN = 5
    SUMSQ = 6
    RMS = 7


class LNMode(enum.IntEnum):
    ONNX = 0
    TADMA = 1


class Dist(enum.IntEnum):
    UNIFORM = 0
    NORMAL = 1
    INDEX = 2


DTYPE_SIZE = {DType.F32: 4, DType.F16: 2, DType.BF16: 2, DType.F64: 8, DType.I64: 8,
              DType.I32: 4, DType.U8: 1, DType.BOOL: 1, DType.I8: 1}

UNARY_OPS = [op for op in Op if op < 32]
BINARY_OPS = [op for op in Op if 32 <= op < 64]
TRANSCENDENTAL = {Op.EXP, Op.LOG, Op.SQRT, Op.SIN, Op.COS, Op.TAN, Op.ASIN, Op.ACOS, Op.ATAN,
                  Op.ASINH, Op.ACOSH, Op.ATANH, Op.ERF, Op.SIGMOID, Op.TANH, Op.GELU}


class TadmaTensor(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("dims", ctypes.c_int64 * MAX_RANK),
        ("strides", ctypes.c_int64 * MAX_RANK),
    ]


class TadmaInstr(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("b", ctypes.c_int32),
        ("c", ctypes.c_int32),
        ("round_dtype", ctypes.c_int32),
        ("imm", ctypes.c_double),
    ]


ROWPROG_MAX_STAGES = 3


class TadmaRowStage(ctypes.Structure):
    """tadma_row_stage: one per-row reduction of an element chain."""
    _fields_ = [
        ("op", ctypes.c_int32),
        ("n_instr", ctypes.c_int32),
        ("n_post", ctypes.c_int32),
        ("acc", ctypes.c_int32),
        ("prog", TadmaInstr * MAX_INSTR),
        ("post", TadmaInstr * MAX_INSTR),
        ("out", TadmaTensor),
    ]


class TadmaRowProgram(ctypes.Structure):
    """tadma_row_program: stages, then the final chain, over a row grid."""
    _fields_ = [
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("n_ins", ctypes.c_int32),
        ("n_stages", ctypes.c_int32),
        ("n_instr", ctypes.c_int32),
        ("compute", ctypes.c_int32),
        ("acc", ctypes.c_int32),
        ("pad", ctypes.c_int32),
        ("ins", TadmaTensor * MAX_INPUTS),
        ("stages", TadmaRowStage * ROWPROG_MAX_STAGES),
        ("prog", TadmaInstr * MAX_INSTR),
        ("out", TadmaTensor),
    ]


def make_tensor(ptr: int | None, dtype: int, shape, strides=None) -> TadmaTensor:
    """Descriptor for a strided view; strides in ELEMENTS (default row-major)."""
    shape = [int(s) for s in shape]
    if len(shape) > MAX_RANK:
        raise ValueError(f"rank {len(shape)} exceeds {MAX_RANK}")
    if strides is None:
        strides, acc = [0] * len(shape), 1
        for d in range(len(shape) - 1, -1, -1):
            strides[d] = acc
            acc *= shape[d]
    t = TadmaTensor()
    t.data = ptr
    t.dtype = int(dtype)
    t.rank = len(shape)
    for d, (n, s) in enumerate(zip(shape, strides)):
        t.dims[d] = n
        t.strides[d] = int(s)
    return t


def instr(op, b=SRC_NONE, c=SRC_NONE, round_dtype=-1, imm=0.0) -> TadmaInstr:
    return TadmaInstr(int(op), int(b), int(c), int(round_dtype), float(imm))


def program(instrs) -> tuple[ctypes.Array, int]:
    arr = (TadmaInstr * max(1, len(instrs)))(*instrs)
    return arr, len(instrs)


# ---- numpy <-> dtype (bf16 is carried as raw uint16) ---------------------------

_NP_OF = {DType.F32: np.float32, DType.F16: np.float16, DType.BF16: np.uint16, DType.F64: np.float64,
          DType.I64: np.int64, DType.I32: np.int32, DType.U8: np.uint8, DType.BOOL: np.bool_,
          DType.I8: np.int8}


def np_dtype(dt: int):
    return _NP_OF[DType(dt)]


def dtype_of_np(a: np.ndarray) -> DType:
    for k, v in _NP_OF.items():
        if a.dtype == np.dtype(v) and k != DType.BF16:
            return k
    if a.dtype == np.uint16:
        return DType.BF16
    raise TypeError(f"no tadma dtype for numpy {a.dtype}")


def host_tensor(a: np.ndarray, dtype: int | None = None) -> TadmaTensor:
    """Descriptor of a host numpy array (strides converted to elements)."""
    dt = DType(dtype) if dtype is not None else dtype_of_np(a)
    es = a.itemsize
    strides = [s // es for s in a.strides]
    return make_tensor(a.ctypes.data if a.size else None, dt, a.shape, strides)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 (raw uint16), NaN kept quiet."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
