"""Leading-axis sharding and the cross-shard reduction, on CPU with gloo
(world_size 2): host logic of the multi-GPU path, no GPU needed.  Rank
failures are made on the host (a rank that raises / never reports)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tadma_b200.shard import Shard, element_offset, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 32, 2048, 2049):
        for world in (1, 2, 3, 4, 8):
            shards = [shard_range(n, r, world) for r in range(world)]
            assert shards[0].start == 0 and shards[-1].stop == n
            for a, b in zip(shards, shards[1:]):
                assert a.stop == b.start
            sizes = [s.size for s in shards]
            assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_shard_generation_offsets_match_full_tensor():
    # a shard generated at its global element offset equals those rows of the full tensor
    from oracle import oracle as O
    from tadma_b200.abi import Dist, DType
    full = O.fill((8, 16), DType.F32, Dist.NORMAL, 0, 1, 0, 1)
    for r in range(4):
        s = shard_range(8, r, 4)
        part = O.fill((s.size, 16), DType.F32, Dist.NORMAL, 0, 1, 0, 1, offset=element_offset(s, 16))
        assert np.array_equal(part, full[s.start:s.stop])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_reduce(rank, world, port, q):
    import torch
    from oracle import oracle as O
    from tadma_b200.abi import Dist, DType, Reduce
    from tadma_b200.shard import allreduce_partials, init_group
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist = init_group("gloo", timeout_s=30, rank=rank, world_size=world)
    s = shard_range(6, rank, world)
    x = O.fill((s.size, 5, 7), DType.F32, Dist.UNIFORM, -1, 1, 0, 3, offset=element_offset(s, 35))
    part = np.zeros((1, 5, 7), np.float32)
    O.reduce(Reduce.SUM, x, 0, part)  # the local slab reduction (oracle stands in for the GPU kernel on CPU)
    t = torch.from_numpy(part.astype(np.float64))
    allreduce_partials(t, "sum")
    mx = torch.from_numpy(x.max(axis=0, keepdims=True).astype(np.float64))
    allreduce_partials(mx, "max")
    q.put((rank, t.numpy(), mx.numpy()))
    dist.destroy_process_group()


def test_cross_shard_reduction_gloo_world2():
    from oracle import oracle as O
    from tadma_b200.abi import Dist, DType
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_reduce, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full = O.fill((6, 5, 7), DType.F32, Dist.UNIFORM, -1, 1, 0, 3)
    for _, s, m in res:
        np.testing.assert_allclose(s[0], full.astype(np.float64).sum(axis=0), rtol=1e-6, atol=1e-6)
        assert np.array_equal(m[0], full.max(axis=0))


def _rank_fail(rank, world, port, q):
    from tadma_b200.shard import RankFailure, init_group, run_checked
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    init_group("gloo", timeout_s=10, rank=rank, world_size=world)
    store = dist.distributed_c10d._get_default_store()

    def step():
        if rank == 1:
            raise ValueError("injected host-side failure")
        return "done"

    try:
        run_checked(step, store, rank, world, "step0", timeout_s=5)
        q.put((rank, "ok"))
    except RankFailure as e:
        q.put((rank, f"peer-failure: {e}"))
    except ValueError as e:
        q.put((rank, f"raised: {e}"))
    # no collective after a failure: every rank leaves between steps
    dist.destroy_process_group()


def test_rank_failure_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fail, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res[1].startswith("raised: injected")
    assert res[0].startswith("peer-failure") and "rank 1 failed" in res[0]


def _rank_silent(rank, world, port, q):
    from tadma_b200.shard import RankFailure, init_group, run_checked
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    init_group("gloo", timeout_s=10, rank=rank, world_size=world)
    store = dist.distributed_c10d._get_default_store()
    if rank == 1:
        q.put((rank, "left"))  # a rank that leaves without reporting
        return
    try:
        run_checked(lambda: 1, store, rank, world, "stepX", timeout_s=2)
        q.put((rank, "ok"))
    except RankFailure as e:
        q.put((rank, f"peer-failure: {e}"))


def test_rank_that_never_reports_times_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_silent, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0].startswith("peer-failure") and "did not report" in res[0]
