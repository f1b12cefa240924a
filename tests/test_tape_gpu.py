"""The header API's ExecutionTape / node layer on the B200: tests/cpp/tape.cu
in "cuda" mode (merged nodes as one header-compiled kernel, trampolines,
user functors, extended lambdas) and the reference's own demo main.cu,
compiled unchanged against include/tadma, each checked against the oracle."""
import os
import subprocess

import pytest

from tests import tape_check

pytestmark = pytest.mark.gpu


def test_tape_program_on_cuda_tensors(tmp_path):
    exe = tape_check.build_tape(str(tmp_path))
    nodes = tape_check.run_tape(exe, "cuda", str(tmp_path))
    # chain: the index node and five operator nodes merge into one kernel,
    # plus the output node; host_lambda: the host-only index node stays
    # apart; transposed: the transposed read is not merged.
    assert nodes == {"chain": 2, "host_lambda": 3, "transposed": 3}
    tape_check.check_outputs(str(tmp_path))


@pytest.mark.skipif(not os.path.exists(tape_check.REF_MAIN_BIN),
                    reason="tests/cpp/_ref/tape_main is built by __graft_entry__.build() where the reference exists")
def test_reference_demo_runs_and_matches_oracle():
    r = subprocess.run([tape_check.REF_MAIN_BIN], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    tape_check.check_reference_main_output(r.stdout)
