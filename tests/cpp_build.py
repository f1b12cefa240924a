"""Builds tests/cpp/conformance.cu against include/tadma (header-only API) and libtadma_b200.so."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_program(name: str, out_dir: str) -> str:
    """nvcc tests/cpp/<name>.cu -> <out_dir>/<name>, linked against libtadma_b200.so."""
    exe = os.path.join(out_dir, name)
    lib_dir = os.path.join(ROOT, "tadma_b200")
    cmd = ["nvcc", "-std=c++20", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "cpp", name + ".cu"),
           "-L", lib_dir, "-ltadma_b200", "-Xlinker", f"-rpath={lib_dir}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{name} build failed:\n{r.stdout}\n{r.stderr}")
    return exe


def build_conformance(out_dir: str) -> str:
    return build_program("conformance", out_dir)
