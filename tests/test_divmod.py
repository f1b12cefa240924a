"""The element-index divider of the CUDA kernels (DivMod in
tadma_b200/csrc/common.cuh), checked on the host: 64-bit and 32-bit magic
quotients against exact division.  CPU only (nvcc host compile, no GPU)."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_divmod_quotients(tmp_path):
    exe = os.path.join(str(tmp_path), "divmod_check")
    src = os.path.join(ROOT, "tests", "cpp", "divmod_check.cu")
    r = subprocess.run(["nvcc", "-std=c++17", "-O2", src, "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr
