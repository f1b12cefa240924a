"""Two GPUs, one process each (NCCL over NVLink): the leading-axis sharded
reduction (shard.reduce_leading_axis_sharded: the local slab reduce with
tadma_b200_reduce, then one all-reduce of the partial) equals the oracle's
reduction of the whole tensor, and each rank's generated slab is exactly its
rows of the full tensor.  Skipped on a box with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch
    import tadma_b200 as tb
    from tadma_b200.abi import Dist
    from tadma_b200.shard import element_offset, init_group, reduce_leading_axis_sharded, shard_range
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist = init_group("nccl", timeout_s=60, rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        B, R, C = 7, 96, 640
        s = shard_range(B, rank, world)
        x = torch.empty((s.size, R, C), dtype=torch.float32, device="cuda")
        tb.fill(x, Dist.UNIFORM, -1.0, 1.0, 0, 5, offset=element_offset(s, R * C))
        out = {}
        for op in ("sum", "max"):
            o = torch.empty((1, R, C), dtype=torch.float32, device="cuda")
            reduce_leading_axis_sharded(x, o, op)
            out[op] = o.cpu().numpy()
        q.put((rank, out, x.cpu().numpy()))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sharded_leading_axis_reduce_nccl_2gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle import oracle as O
    from tadma_b200.abi import Dist, DType
    from tadma_b200.shard import shard_range
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out, slab = q.get(timeout=300)
        res[r] = (out, slab)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = O.fill((7, 96, 640), DType.F32, Dist.UNIFORM, -1.0, 1.0, 0, 5)
    for r in range(2):
        s = shard_range(7, r, 2)
        assert np.array_equal(res[r][1], full[s.start:s.stop])
        np.testing.assert_allclose(res[r][0]["sum"][0], full.astype(np.float64).sum(axis=0), rtol=0, atol=1e-5 * 7)
        assert np.array_equal(res[r][0]["max"][0], full.max(axis=0))
