"""The header API's ExecutionTape / node layer on host tensors (no GPU):
tests/cpp/tape.cu in "cpu" mode against the oracle, and the reference's own
demo (main.cu) compiling unchanged against include/tadma."""
import os

import pytest

from tests import tape_check


def test_tape_program_on_host_tensors(tmp_path):
    exe = tape_check.build_tape(str(tmp_path))
    nodes = tape_check.run_tape(exe, "cpu", str(tmp_path))
    # Host nodes are never merged (merging exists to fuse device kernels).
    assert nodes == {"chain": 7, "host_lambda": 4, "transposed": 3}
    tape_check.check_outputs(str(tmp_path))


@pytest.mark.skipif(not os.path.exists(os.path.join(tape_check.reference_dir(), "main.cu")),
                    reason="reference checkout not present (set TADMA_REFERENCE)")
def test_reference_demo_compiles_unchanged():
    exe = tape_check.build_reference_main()
    assert exe and os.path.exists(exe)
