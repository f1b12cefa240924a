"""Prepared C-ABI calls captured into a CUDA graph (the launch-bound
config-1 step: t = A + b, then the row sum with exp as its pre-op) replay
with the same results as the eager calls and the oracle.  The kernels are
launched with programmatic dependent launch, so the graph carries
programmatic edges between them."""
import numpy as np
import pytest

import tadma_b200 as tb
from oracle import oracle as O
from tadma_b200.abi import Compute, Dist, DType, Op, Reduce, instr, make_tensor
from tests.helpers import gen

pytestmark = pytest.mark.gpu


def test_graph_replay_of_prepared_calls():
    import torch
    R, C = 64, 128
    A = torch.from_numpy(gen((R, C), DType.F32, Dist.NORMAL, 0, 1, 1)).cuda()
    b = torch.from_numpy(gen((C,), DType.F32, Dist.NORMAL, 0, 1, 2)).cuda()
    t = torch.empty_like(A)
    y = torch.full((R, 1), -1.0, dtype=torch.float32, device="cuda")
    bv = make_tensor(b.data_ptr(), DType.F32, [R, C], [0, 1])
    side = torch.cuda.Stream()
    calls = [tb.prepare_eltwise(t, [A, bv], [instr(Op.ADD, b=1)], Compute.F32, stream=side),
             tb.prepare_reduce(Reduce.SUM, t, -1, y, Op.EXP, stream=side)]
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for c in calls:
            c()
    side.synchronize()
    eager = y.cpu().numpy().copy()
    y.fill_(-1.0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        for c in calls:
            c()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert np.array_equal(got, eager)
    ref = np.zeros((R, 1), np.float32)
    assert O.reduce(Reduce.SUM, (A.cpu().numpy() + b.cpu().numpy()).astype(np.float32), -1, ref, Op.EXP) == 0
    np.testing.assert_allclose(got, ref, rtol=1e-5 * np.sqrt(C))
    del g
