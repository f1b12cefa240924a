"""Weight-file constructor on host tensors (no GPU): every member of a file in
the generator's layout reads back byte for byte."""
from tests import weights_check


def test_weight_file_host_tensors(tmp_path):
    weights_check.run(str(tmp_path), cuda=False)
