"""Shared steps of the weight-file tests: a file in the generator's layout
(raw tensors back to back, cppgen.py:111-116) of random bytes, loaded by
tests/cpp/weights.cu and compared byte for byte."""
import os
import subprocess

import numpy as np

from tests.cpp_build import build_program

MEMBERS = [("a", 3 * 5 * 7 * 2), ("b", 8192 * 1536 * 4), ("c", 129 * 8), ("d", 1000 * 3 * 2), ("e", 17 * 8),
           ("f", 4096 * 1024 * 4)]


def run(tmp: str, cuda: bool) -> None:
    exe = build_program("weights", tmp)
    blob = np.random.default_rng(5).integers(0, 256, sum(n for _, n in MEMBERS), dtype=np.uint8)
    path = os.path.join(tmp, "model.bin")
    blob.tofile(path)
    r = subprocess.run([exe, path, tmp] + (["cuda"] if cuda else []), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "weights ok" in r.stdout
    off = 0
    for name, n in MEMBERS:
        for ext in ("cpu", "cuda") if cuda else ("cpu",):
            got = np.fromfile(os.path.join(tmp, f"{name}.{ext}"), dtype=np.uint8)
            assert np.array_equal(got, blob[off:off + n]), (name, ext)
        off += n
