"""tadma_b200.pipeline.RowPipeline: host-buffer execution of a row op with the
upload, per-chunk C-ABI calls and download overlapped on three streams gives
the same bytes as one call on device buffers (and as the oracle)."""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import SRC_IMM, Compute, Dist, DType, Op, instr, make_tensor
from tests.helpers import gen, ulp_diff

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,chunks", [(1000, 7), (64, 16), (5, 8)])
def test_row_pipeline_matches_oracle(rows, chunks):
    import torch
    C = 256
    x = gen((rows, C), DType.BF16, Dist.NORMAL, 0, 1, 31)
    b = gen((C,), DType.BF16, Dist.NORMAL, 0, 0.1, 32)
    prog = [instr(Op.MUL, b=SRC_IMM, imm=0.5, round_dtype=DType.F32), instr(Op.ADD, b=1, round_dtype=DType.F32),
            instr(Op.GELU, round_dtype=DType.F32)]
    xh = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory()
    bh = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd, bd, yd = torch.empty_like(xh, device="cuda"), torch.empty_like(bh, device="cuda"), torch.empty_like(xh, device="cuda")

    def make_call(lo, hi, st):
        bv = make_tensor(bd.data_ptr(), DType.BF16, [hi - lo, C], [0, 1])
        return tb.prepare_eltwise(yd[lo:hi], [xd[lo:hi], bv], prog, Compute.F32, stream=st)

    from tadma_b200.pipeline import RowPipeline
    pipe = RowPipeline(rows, chunks, uploads=[(xh, xd)], downloads=[(yd, yh)], make_call=make_call, once=[(bh, bd)])
    s = torch.cuda.current_stream()
    for _ in range(2):
        yh.zero_()
        pipe(s)
        s.synchronize()
    got = yh.view(torch.int16).numpy().view(np.uint16)
    ref = np.zeros_like(x)
    rc = O.eltwise(ref, [x, np.broadcast_to(b, (rows, C))], prog, Compute.F32, in_dtypes=[DType.BF16, DType.BF16],
                   out_dtype=DType.BF16)
    assert rc == 0
    assert ulp_diff(got, ref, DType.BF16).max() <= 1  # fast gelu on a 16-bit output: <= 1 bf16 ulp
