"""Drop-in check of the generated-code calling convention: the reference's
own generated graph (scripts/generated.cu of OgnianM/TADMA, a BERT model
emitted by its onnx2tadma/cppgen scripts) compiles unchanged against
include/tadma, with tadma/Tadma.hpp force-included (the checked-in file has
lost its #include line), and its infer<batch, sequence>() instantiates.
Compile-only; skipped when the reference checkout is not present."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The reference checkout: $TADMA_REFERENCE, else ../reference beside the repository.
REFERENCE = os.environ.get("TADMA_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
GENERATED = os.path.join(REFERENCE, "scripts", "generated.cu")


@pytest.mark.skipif(not os.path.exists(GENERATED), reason="reference checkout not present (set TADMA_REFERENCE)")
def test_reference_generated_graph_compiles_unchanged(tmp_path):
    wrapper = tmp_path / "instantiate.cu"
    seq = "Tensor<int64_t, ALLOCATOR, Sequence<(int64_t)1, (int64_t)8>>"
    wrapper.write_text(f'#include "{GENERATED}"\n'
                       f"template auto Model::infer<1, 8>({seq}, {seq}, {seq});\n")
    cmd = ["nvcc", "-std=c++20", "-gencode", "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "include"),
           "-include", "tadma/Tadma.hpp", "-x", "cu", "-c", str(wrapper), "-o", str(tmp_path / "generated.o")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
