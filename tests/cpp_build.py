"""Builds the C++ test programs (tests/cpp/*.cu) against include/tadma (header-only API) and libtadma_b200.so."""
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


def reference_dir() -> str:
    """The reference checkout: $TADMA_REFERENCE, else ../reference beside the repository."""
    return os.environ.get("TADMA_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))


REF_MAIN_BIN = os.path.join(ROOT, "tests", "cpp", "_ref", "tape_main")


def build_reference_main() -> str | None:
    """Compiles the reference's own demo (main.cu: an ExecutionTape of an
    index_to_value node and seven operator nodes, Optimize, Evaluate, print)
    unchanged against include/tadma.  The file is copied to a scratch
    directory first, because its `#include "include/tadma/Tadma.hpp"` would
    otherwise find the reference's headers next to it.  Returns the binary
    (tests/cpp/_ref/tape_main, git-ignored; it travels with the repository
    to the GPU box) or None without a reference checkout."""
    src = os.path.join(reference_dir(), "main.cu")
    if not os.path.exists(src):
        return None
    import shutil
    import tempfile
    os.makedirs(os.path.dirname(REF_MAIN_BIN), exist_ok=True)
    lib_dir = os.path.join(ROOT, "tadma_b200")
    with tempfile.TemporaryDirectory() as tmp:
        shutil.copyfile(src, os.path.join(tmp, "main.cu"))
        cmd = ["nvcc", "-std=c++20", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-I", ROOT,
               os.path.join(tmp, "main.cu"), "-L", lib_dir, "-ltadma_b200", "-Xlinker", f"-rpath={lib_dir}",
               "-o", REF_MAIN_BIN]
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    return REF_MAIN_BIN
