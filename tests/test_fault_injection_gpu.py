"""Host-side fault injection: TADMA_B200_FAIL_ALLOC=1 makes every device
workspace allocation fail as on an exhausted device, before any CUDA call.
A reduction that needs a workspace (a long row split across CTAs) then
returns TADMA_ERR_CUDA with the allocator's message, launches nothing and
leaves its output untouched.  The CUDA context stays usable: the
no-allocation entry point, reductions that need no workspace, and the same
call once the variable is cleared all succeed.  No GPU fault is involved."""
import ctypes

import numpy as np
import pytest

import tadma_b200 as tb
from tadma_b200.abi import Dist, DType, Reduce, Status
from tests.helpers import empty_dev

pytestmark = pytest.mark.gpu


def test_injected_workspace_allocation_failure(monkeypatch):
    import torch
    x = empty_dev((2, 1 << 21), DType.F32)
    tb.fill(x, Dist.NORMAL, 0.0, 1.0, seed=0, stream_id=31)
    ref = x.double().sum(-1)
    out = empty_dev((2,), DType.F32)
    out.fill_(7.0)
    torch.cuda.synchronize()

    monkeypatch.setenv("TADMA_B200_FAIL_ALLOC", "1")
    with pytest.raises(tb.TadmaError) as err:
        tb.reduce(Reduce.SUM, x, -1, out)
    assert err.value.code == Status.ERR_CUDA
    assert "workspace" in str(err.value) and "memory" in str(err.value).lower()
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing launched

    # entry points that allocate nothing are unaffected
    small = empty_dev((64, 1), DType.F32)
    tb.reduce(Reduce.SUM, x[:, :4096].contiguous().view(64, 128), -1, small)
    i, o = tb.desc(x), tb.desc(out)
    rc = tb.lib().tadma_b200_reduce_noalloc(int(Reduce.SUM), ctypes.byref(i), -1, 0, ctypes.byref(o),
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, tb.lib().tadma_b200_last_error()
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.double().cpu().numpy(), ref.cpu().numpy(), rtol=1e-5 * np.sqrt(1 << 21))

    monkeypatch.delenv("TADMA_B200_FAIL_ALLOC")
    out.fill_(7.0)
    tb.reduce(Reduce.SUM, x, -1, out)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.double().cpu().numpy(), ref.cpu().numpy(), rtol=1e-5 * np.sqrt(1 << 21))
    assert tb.error_flags() == 0
