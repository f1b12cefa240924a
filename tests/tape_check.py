"""Checks of tests/cpp/tape.cu's outputs (CPU and GPU runs) against the oracle.

The chain a -> 3a -> 3a + 1.5 -> (3a + 1.5) a -> sigmoid -> - 3a is the
oracle's element-wise chain on the program's own `a` (fp32 compute, rounded
after every op); the device's sigmoid (expf-based) is within 4 ulp of the
oracle's.  Exact cases (host lambda, transposed copy, functor and lambda
nodes) are compared with an explicit tolerance each."""
import os
import re
import subprocess

import numpy as np

from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, DType, Op, instr
from tests.cpp_build import REF_MAIN_BIN, ROOT, build_reference_main, reference_dir  # noqa: F401
from tests.helpers import ulp_diff


def build_tape(out_dir: str) -> str:
    exe = os.path.join(out_dir, "tape")
    lib_dir = os.path.join(ROOT, "tadma_b200")
    cmd = ["nvcc", "-std=c++20", "-O2", "--extended-lambda", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "cpp", "tape.cu"),
           "-L", lib_dir, "-ltadma_b200", "-Xlinker", f"-rpath={lib_dir}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    return exe


def run_tape(exe: str, mode: str, out_dir: str) -> dict:
    r = subprocess.run([exe, mode, out_dir], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "tape ok" in r.stdout and "extended lambda ok" in r.stdout
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"nodes (\w+) (\d+)", r.stdout)}


def check_outputs(out_dir: str) -> None:
    def ld(name, shape):
        return np.fromfile(os.path.join(out_dir, name + ".bin"), dtype=np.float32).reshape(shape)

    a, f = ld("chain_a", (64, 96)), ld("chain_f", (64, 96))
    i = np.arange(64 * 96, dtype=np.float32).reshape(64, 96)
    assert ulp_diff(a, np.cos(np.float32(0.37) * i), DType.F32).max() <= 2
    b = np.zeros_like(a)
    assert O.eltwise(b, [a], [instr(Op.MUL, b=SRC_IMM, imm=3.0, round_dtype=DType.F32)], Compute.F32) == 0
    ref = np.zeros_like(a)
    prog = [instr(Op.ADD, b=SRC_IMM, imm=1.5, round_dtype=DType.F32), instr(Op.MUL, b=1, round_dtype=DType.F32),
            instr(Op.SIGMOID, round_dtype=DType.F32), instr(Op.SUB, b=0, round_dtype=DType.F32)]
    assert O.eltwise(ref, [b, a], prog, Compute.F32) == 0
    # f = sigmoid(.) - 3a: compare within 4 ulp of the larger operand's scale.
    assert np.abs(f - ref).max() <= 4 * np.spacing(np.maximum(np.abs(ref), np.abs(b))).max()

    c = ld("host_lambda_c", (50, 40))
    j = np.arange(2000, dtype=np.float32).reshape(50, 40)
    assert np.array_equal(c, -((j * np.float32(0.5) - np.float32(7)) * np.float32(2)))

    p, q = ld("transposed_p", (48, 80)), ld("transposed_q", (80, 48))
    assert np.array_equal(p, ((np.arange(48 * 80) % 13) - 6).astype(np.float32).reshape(48, 80))
    assert np.array_equal(q, p.T * np.float32(2))

    x, y, z, w = ld("fma_x", (32, 256)), ld("fma_y", (256,)), ld("fma_z", (32, 256)), ld("lambda_w", (32, 256))
    want = np.zeros_like(z)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=2.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32)]
    assert O.eltwise(want, [x, np.broadcast_to(y, x.shape)], prog, Compute.F32) == 0
    # The device may fuse a * x + y into one FMA: it then skips the product's
    # rounding, a difference of at most half an ulp of a * x (plus the sum's).
    prod = np.abs(np.float32(2.5) * x)
    assert np.all(np.abs(z - want) <= np.spacing(prod) + np.spacing(np.abs(want)))
    want = np.zeros_like(w)
    prog = [instr(Op.MUL, b=0, round_dtype=DType.F32), instr(Op.SUB, b=SRC_IMM, imm=1.0, round_dtype=DType.F32)]
    assert O.eltwise(want, [x], prog, Compute.F32) == 0
    assert np.all(np.abs(w - want) <= np.spacing(x * x) + np.spacing(np.abs(want)))


def check_reference_main_output(text: str) -> None:
    """main.cu prints t8 = tanh(t5 * t3) over a 10 x 10 tensor, with
    t1 = cos(i) (i the flat index), t3 = 5 t1 - 5, t5 = -(t3 / pi), every step
    in fp32.  The oracle evaluates the same chain from t1 = cos(i) rounded to
    fp32; tanh and cos are within a few fp32 ulps of each other there, and the
    print keeps 6 significant digits."""
    vals = np.array([float(v) for v in re.findall(r"-?\d+(?:\.\d+)?(?:e[-+]?\d+)?", text)], dtype=np.float64)
    assert vals.size == 100, (vals.size, text[:400])
    t1 = np.cos(np.arange(100, dtype=np.float64)).astype(np.float32).reshape(10, 10)
    t3 = np.zeros_like(t1)
    assert O.eltwise(t3, [t1], [instr(Op.MUL, b=SRC_IMM, imm=5.0, round_dtype=DType.F32),
                                instr(Op.SUB, b=SRC_IMM, imm=5.0, round_dtype=DType.F32)], Compute.F32) == 0
    t8 = np.zeros_like(t1)
    pi32 = float(np.float32(np.pi))
    prog = [instr(Op.DIV, b=SRC_IMM, imm=pi32, round_dtype=DType.F32), instr(Op.NEG, round_dtype=DType.F32),
            instr(Op.MUL, b=0, round_dtype=DType.F32), instr(Op.TANH, round_dtype=DType.F32)]
    assert O.eltwise(t8, [t3], prog, Compute.F32) == 0
    np.testing.assert_allclose(vals.reshape(10, 10), t8.astype(np.float64), rtol=2e-5, atol=2e-6)
