"""The header-only Tensor API (include/tadma) compiles and links against
libtadma_b200.so with nvcc -std=c++20 for sm_100a (no GPU needed)."""
from tests.cpp_build import build_conformance


def test_conformance_program_builds(tmp_path):
    exe = build_conformance(str(tmp_path))
    assert exe.endswith("conformance")


def test_generated_blocks_program_builds(tmp_path):
    # generated-code statements with ConstexprHolder operands, deferred evaluation
    from tests.cpp_build import build_program
    assert build_program("fusion", str(tmp_path)).endswith("fusion")


def test_allocator_fault_injection_throws(tmp_path):
    # TADMA_B200_FAIL_ALLOC=1: the header API's device allocator throws
    # std::runtime_error before calling CUDA (runs without a GPU).
    import subprocess
    from tests.cpp_build import build_program
    exe = build_program("alloc_fault", str(tmp_path))
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "caught: out of memory" in r.stdout
    assert "empty tensor ok" in r.stdout
