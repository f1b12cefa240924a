"""C-ABI conformance without a GPU: the library loads, exports every entry
point declared in include/tadma_b200.h, the Python mirror (tadma_b200.abi)
matches the header's constants, and host-side validation rejects bad
descriptors before any CUDA call."""
import ctypes
import os
import re

import pytest

import tadma_b200 as tb
from tadma_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tadma_b200.h")


def header_text():
    with open(HEADER) as f:
        return f.read()


def test_library_loads_and_exports_every_declared_symbol():
    L = tb.lib()
    declared = set(re.findall(r"\b(tadma_b200_\w+)\s*\(", header_text()))
    assert declared, "no entry points found in the header"
    missing = [s for s in sorted(declared) if not hasattr(L, s)]
    assert not missing, f"not exported: {missing}"
    assert set(tb.EXPORTS) <= declared
    assert "sm_100a" in tb.version()


def test_enums_match_header():
    text = header_text()
    consts = {m.group(1): int(m.group(2)) for m in re.finditer(r"\b(TADMA_[A-Z0-9_]+)\s*=\s*(-?\d+)", text)}
    defines = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+(TADMA_[A-Z0-9_]+)\s+\(?(-?\d+)\)?", text)}
    for e, prefix in ((abi.DType, "TADMA_"), (abi.Op, "TADMA_OP_"), (abi.Reduce, "TADMA_REDUCE_"),
                      (abi.Compute, "TADMA_COMPUTE_"), (abi.Dist, "TADMA_DIST_")):
        for m in e:
            assert consts[prefix + m.name] == int(m), (prefix + m.name)
    assert consts["TADMA_LN_ONNX"] == abi.LNMode.ONNX and consts["TADMA_LN_TADMA"] == abi.LNMode.TADMA
    for m in abi.Status:
        name = "TADMA_OK" if m.name == "OK" else "TADMA_" + m.name
        assert consts[name] == int(m)
    assert defines["TADMA_MAX_RANK"] == abi.MAX_RANK
    assert defines["TADMA_MAX_INPUTS"] == abi.MAX_INPUTS
    assert defines["TADMA_MAX_INSTR"] == abi.MAX_INSTR
    assert defines["TADMA_SRC_IMM"] == abi.SRC_IMM
    assert defines["TADMA_ROWPROG_MAX_STAGES"] == abi.ROWPROG_MAX_STAGES
    assert ctypes.sizeof(abi.TadmaTensor) == 8 + 4 + 4 + 8 * 8 * 2
    assert ctypes.sizeof(abi.TadmaInstr) == 24
    # tadma_row_stage / tadma_row_program: natural alignment, no padding beyond the declared fields
    assert ctypes.sizeof(abi.TadmaRowStage) == 16 + 2 * 16 * 24 + 144
    assert ctypes.sizeof(abi.TadmaRowProgram) == 16 + 24 + 6 * 144 + 3 * ctypes.sizeof(abi.TadmaRowStage) + 16 * 24 + 144


def test_row_program_validation_needs_no_gpu():
    L = tb.lib()
    fake = 0x1000
    rp = abi.TadmaRowProgram()
    rp.rows, rp.cols, rp.n_ins, rp.n_stages, rp.n_instr, rp.compute = 8, 64, 1, 0, 0, int(abi.Compute.F32)
    rp.ins[0] = abi.make_tensor(fake, abi.DType.F32, [8, 64])
    rp.out = abi.make_tensor(fake, abi.DType.F32, [8, 64])
    rp.compute = int(abi.Compute.F64)
    assert L.tadma_b200_row_program(ctypes.byref(rp), None) == abi.Status.ERR_UNSUPPORTED
    rp.compute = int(abi.Compute.F32)
    rp.n_stages = 4
    assert L.tadma_b200_row_program(ctypes.byref(rp), None) == abi.Status.ERR_INVALID
    rp.n_stages = 1
    rp.stages[0].op = int(abi.Reduce.ARGMAX)
    rp.stages[0].out = abi.make_tensor(fake, abi.DType.F32, [8])
    assert L.tadma_b200_row_program(ctypes.byref(rp), None) == abi.Status.ERR_UNSUPPORTED
    rp.stages[0].op = int(abi.Reduce.MEAN)
    rp.stages[0].n_instr = 1
    rp.stages[0].prog[0] = abi.instr(abi.Op.SUB, b=1)  # a stage reads earlier stages only
    assert L.tadma_b200_row_program(ctypes.byref(rp), None) == abi.Status.ERR_INVALID
    rp.stages[0].n_instr = 0
    rp.ins[0] = abi.make_tensor(fake, abi.DType.F32, [8, 64], [64, 2])  # column stride 2
    assert L.tadma_b200_row_program(ctypes.byref(rp), None) == abi.Status.ERR_UNSUPPORTED
    rp.ins[0] = abi.make_tensor(fake, abi.DType.F32, [8, 66])
    rp.cols = 66
    rp.out = abi.make_tensor(fake, abi.DType.F32, [8, 66])
    assert L.tadma_b200_row_program(ctypes.byref(rp), None) == abi.Status.ERR_UNSUPPORTED  # 66 fp32: not 16-byte rows


def test_dtype_sizes():
    L = tb.lib()
    for dt, n in abi.DTYPE_SIZE.items():
        assert L.tadma_b200_dtype_size(int(dt)) == n
    assert L.tadma_b200_dtype_size(99) == 0


def _rc(fn, *args):
    return fn(*args)


def test_host_validation_needs_no_gpu():
    L = tb.lib()
    P = ctypes.byref
    fake = 0x1000  # never dereferenced: every call below fails validation first
    out = abi.make_tensor(fake, abi.DType.F32, [4, 4])
    bad_rank = abi.make_tensor(fake, abi.DType.F32, [1] * 8)
    bad_rank.rank = 9
    x = abi.make_tensor(fake, abi.DType.F32, [4, 5])
    prog, n = abi.program([abi.instr(abi.Op.NEG)])
    ins = (abi.TadmaTensor * 1)(x)
    assert L.tadma_b200_eltwise(P(out), ins, 1, prog, n, -1, None) == abi.Status.ERR_INVALID
    assert b"broadcastable" in L.tadma_b200_last_error()
    assert L.tadma_b200_eltwise(P(bad_rank), None, 0, prog, n, -1, None) == abi.Status.ERR_INVALID
    assert L.tadma_b200_eltwise(P(out), None, 5, prog, n, -1, None) == abi.Status.ERR_INVALID
    badop, n2 = abi.program([abi.instr(77)])
    assert L.tadma_b200_eltwise(P(out), None, 0, badop, n2, -1, None) == abi.Status.ERR_INVALID
    exp_i64, n3 = abi.program([abi.instr(abi.Op.EXP)])
    oi = abi.make_tensor(fake, abi.DType.I64, [4])
    ii = (abi.TadmaTensor * 1)(abi.make_tensor(fake, abi.DType.I64, [4]))
    assert L.tadma_b200_eltwise(P(oi), ii, 1, exp_i64, n3, int(abi.Compute.I64), None) == abi.Status.ERR_UNSUPPORTED
    # reduce: axis / out-shape / argmax dtype checks
    r_out = abi.make_tensor(fake, abi.DType.F32, [4, 1])
    assert L.tadma_b200_reduce(0, P(out), 2, 0, P(r_out), None) == abi.Status.ERR_INVALID
    assert L.tadma_b200_reduce(int(abi.Reduce.ARGMAX), P(out), 1, 0, P(r_out), None) == abi.Status.ERR_INVALID
    assert L.tadma_b200_reduce(0, P(out), 1, 0, P(abi.make_tensor(fake, abi.DType.F32, [4, 2])), None) == abi.Status.ERR_INVALID
    # gather: ids dtype and out shape
    ids_f = abi.make_tensor(fake, abi.DType.F32, [3])
    g_out = abi.make_tensor(fake, abi.DType.F32, [3, 4])
    assert L.tadma_b200_gather(P(out), 0, P(ids_f), None, P(g_out), None) == abi.Status.ERR_INVALID
    ids = abi.make_tensor(fake, abi.DType.I64, [3])
    assert L.tadma_b200_gather(P(out), 0, P(ids), None, P(abi.make_tensor(fake, abi.DType.F32, [3, 5])), None) == abi.Status.ERR_INVALID
    # layer norm: mode and gamma length
    assert L.tadma_b200_layer_norm(P(out), -1, None, None, ctypes.c_double(1e-5), 7, P(out), None) == abi.Status.ERR_INVALID
    gam = abi.make_tensor(fake, abi.DType.F32, [5])
    assert L.tadma_b200_layer_norm(P(out), -1, P(gam), None, ctypes.c_double(1e-5), 0, P(out), None) == abi.Status.ERR_INVALID
    # reduce_chain: operand count, broadcast, axis, out shape, argmax dtype, empty max
    rc_ins = (abi.TadmaTensor * 2)(abi.make_tensor(fake, abi.DType.F32, [4, 5]),
                                   abi.make_tensor(fake, abi.DType.F32, [1, 5], [0, 1]))
    add, na = abi.program([abi.instr(abi.Op.ADD, b=1)])
    rc_out = abi.make_tensor(fake, abi.DType.F32, [4, 1])
    RC = L.tadma_b200_reduce_chain
    assert RC(0, rc_ins, 0, add, na, -1, -1, P(rc_out), None) == abi.Status.ERR_INVALID          # no operand
    assert RC(0, rc_ins, 2, add, na, -1, 2, P(rc_out), None) == abi.Status.ERR_INVALID           # axis
    assert RC(0, rc_ins, 2, add, na, -1, -1, P(abi.make_tensor(fake, abi.DType.F32, [4, 2])), None) == abi.Status.ERR_INVALID
    assert RC(int(abi.Reduce.ARGMAX), rc_ins, 2, add, na, -1, -1, P(rc_out), None) == abi.Status.ERR_INVALID
    bad_b = (abi.TadmaTensor * 2)(abi.make_tensor(fake, abi.DType.F32, [4, 5]), abi.make_tensor(fake, abi.DType.F32, [3, 5]))
    assert RC(0, bad_b, 2, add, na, -1, -1, P(rc_out), None) == abi.Status.ERR_INVALID          # dims do not broadcast
    sel2, ns = abi.program([abi.instr(abi.Op.ADD, b=2)])
    assert RC(0, rc_ins, 2, sel2, ns, -1, -1, P(rc_out), None) == abi.Status.ERR_INVALID        # selector out of range
    empty = (abi.TadmaTensor * 1)(abi.make_tensor(None, abi.DType.F32, [4, 0]))
    assert RC(int(abi.Reduce.MAX), empty, 1, add, 0, -1, -1, P(rc_out), None) == abi.Status.ERR_INVALID
    # fill: distribution / dtype pairing
    assert L.tadma_b200_fill(P(out), 2, ctypes.c_double(0), ctypes.c_double(10), 0, 0, 0, None) == abi.Status.ERR_INVALID
    assert L.tadma_b200_fill(P(out), 9, ctypes.c_double(0), ctypes.c_double(1), 0, 0, 0, None) == abi.Status.ERR_INVALID


def test_zero_element_calls_are_noops():
    L = tb.lib()
    z = abi.make_tensor(None, abi.DType.F32, [0, 4])
    prog, n = abi.program([abi.instr(abi.Op.NEG)])
    ins = (abi.TadmaTensor * 1)(z)
    assert L.tadma_b200_eltwise(ctypes.byref(z), ins, 1, prog, n, -1, None) == 0
