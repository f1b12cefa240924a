"""The header-only Tensor API (include/tadma) compiles and links against
libtadma_b200.so with nvcc -std=c++20 for sm_100a (no GPU needed)."""
from tests.cpp_build import build_conformance


def test_conformance_program_builds(tmp_path):
    exe = build_conformance(str(tmp_path))
    assert exe.endswith("conformance")
