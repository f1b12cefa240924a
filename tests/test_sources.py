"""Source-level invariants of the CUDA kernels (CPU, no GPU needed).

Every kernel is launched with programmatic stream serialisation
(launch_pdl), so it may start while the previous kernel of its stream is
still running; each one must therefore call pdl_begin() (which waits for the
previous grid) before it touches global memory, i.e. as its first statement.
"""
import os
import re

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tadma_b200", "csrc")


def _sources():
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cuh")):
            with open(os.path.join(CSRC, f)) as fh:
                yield f, fh.read()


def test_every_kernel_waits_for_its_predecessor_first():
    found = 0
    for name, src in _sources():
        for m in re.finditer(r"__global__ void [^{;]*?(\w+_kernel)\([^{;]*\)\s*\{", src):
            found += 1
            body = src[m.end():m.end() + 400]
            first = [ln.strip() for ln in body.splitlines() if ln.strip() and not ln.strip().startswith("//")][0]
            assert first == "pdl_begin();", f"{name}: {m.group(1)} does not start with pdl_begin()"
    assert found >= 15


def test_no_triple_chevron_launches():
    for name, src in _sources():
        code = "\n".join(ln for ln in src.splitlines() if not ln.strip().startswith("//"))
        assert "<<<" not in code, f"{name}: launch without launch_pdl"
