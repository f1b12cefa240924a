"""Deferred evaluation behind the eager API, on unchanged generated-code
statements (tests/cpp/fusion.cu): the ONNX LayerNorm decomposition of
scripts/generated.cu (mean, -, pow, mean, + eps, sqrt, /, *, +) runs in 1
launch (a row program) instead of 9, and the erf GELU (/, erf, +, *, *) in 1 instead of 5,
with the same bits as the eager calls; both against the oracle."""
import os
import re
import subprocess

import numpy as np
import pytest

from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, DType, LNMode, Op, instr
from tests.cpp_build import build_program
from tests.helpers import ulp_diff

pytestmark = pytest.mark.gpu


def test_generated_blocks_fuse_with_eager_bits(tmp_path):
    exe = build_program("fusion", str(tmp_path))
    r = subprocess.run([exe, "check", str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    launches = {(m.group(1), m.group(2)): int(m.group(3)) for m in re.finditer(r"launches (\w+) (\w+) (\d+)", r.stdout)}
    # the LayerNorm's two reductions and its tail: one row program
    assert launches[("ln", "eager")] == 9 and launches[("ln", "deferred")] == 1, launches
    assert launches[("gelu", "eager")] == 5 and launches[("gelu", "deferred")] == 1, launches

    def ld(name, shape):
        return np.fromfile(os.path.join(tmp_path, name + ".bin"), dtype=np.float32).reshape(shape)

    x, g, b = ld("x", (512, 768)), ld("gamma", (768,)), ld("beta", (768,))
    for case in ("ln", "gelu"):
        assert np.array_equal(ld(case + "_deferred", (512, 768)), ld(case + "_eager", (512, 768))), case
    # LayerNorm, ONNX form sqrt(var + eps): fp32 statistics in another fold order
    ref = np.zeros_like(x)
    assert O.layer_norm(x, -1, g, b, 1e-12, LNMode.ONNX, ref) == 0
    got = ld("ln_deferred", (512, 768))
    assert np.abs(got - ref).max() <= 1e-5 * np.sqrt(768) * np.abs(ref).max()
    # erf GELU: + - * / round once; erff is within 2 ulp of the oracle's erf
    ref = np.zeros_like(x)
    prog = [instr(Op.DIV, b=SRC_IMM, imm=float(np.float32(1.4142135381698608)), round_dtype=DType.F32),
            instr(Op.ERF, round_dtype=DType.F32), instr(Op.ADD, b=SRC_IMM, imm=1.0, round_dtype=DType.F32),
            instr(Op.MUL, b=0, round_dtype=DType.F32), instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32)]
    assert O.eltwise(ref, [x], prog, Compute.F32) == 0
    got = ld("gelu_deferred", (512, 768))
    assert np.all(np.abs(got - ref) <= 4 * np.spacing(np.maximum(np.abs(ref), np.abs(x) * np.float32(0.5))))
