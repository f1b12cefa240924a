"""The shared-divisor division of the LayerNorm tail (tadma_b200/csrc/kdiv.cuh:
reciprocal once, then two fused-multiply-add corrections), checked on the host
against IEEE division for every fp32 dividend of its range and 40 divisors,
plus 2^28 pseudo-random pairs.  CPU only (nvcc host compile, OpenMP)."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shared_divisor_quotients_are_correctly_rounded(tmp_path):
    exe = os.path.join(str(tmp_path), "kdiv_check")
    src = os.path.join(ROOT, "tests", "cpp", "kdiv_check.cu")
    r = subprocess.run(["nvcc", "-std=c++17", "-O3", "-Xcompiler", "-fopenmp,-mfma,-ffp-contract=off,-O3", src, "-o",
                        exe, "-lgomp"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr
