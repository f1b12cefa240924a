"""Weight-file constructor on CUDA tensors: members stream through the pinned
staging ring (one member spans four slots and wraps the ring, one fills a slot
exactly, the small ones start at unaligned file offsets) and read back byte
for byte."""
import pytest

from tests import weights_check

pytestmark = pytest.mark.gpu


def test_weight_file_cuda_tensors(tmp_path):
    weights_check.run(str(tmp_path), cuda=True)
