"""Leading-axis (batch) sharding across the GPUs of one box.

Every config of the hot path is independent along its leading axis, so each
rank owns a contiguous slab of it and runs the same kernels on its own HBM:
no collective on the data path.  The only exchange is a reduction ACROSS the
sharded axis (e.g. sum over axis 0 of X[32, 4096, 4096] split by batch): each
rank reduces its slab with tadma_b200_reduce, then one all-reduce (NCCL over
NVLink on GPUs, gloo on CPU) combines the partials.

Failure handling is host-side: the process group is created with a short
timeout so a rank that dies or never joins turns a peer's next collective into
an error instead of a hang; `run_checked` wraps a rank's step and reports the
first failure to every rank through the store before any further collective.
"""
from __future__ import annotations

import datetime
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int  # first index of this rank's slab on the leading axis
    stop: int   # one past the last index

    @property
    def size(self) -> int:
        return self.stop - self.start


def shard_range(n: int, rank: int, world: int) -> Shard:
    """Contiguous split of [0, n) into `world` slabs; the first n % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n < 0:
        raise ValueError("negative extent")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    size = base + (1 if rank < extra else 0)
    return Shard(rank, world, start, start + size)


def element_offset(shard: Shard, row_elems: int) -> int:
    """Global element index of the shard's first element (the seeded generator's
    `offset`, so a shard generates exactly the rows of the full tensor)."""
    return shard.start * row_elems


def init_group(backend: str, timeout_s: float = 60.0, **kw):
    """torch.distributed.init_process_group with a bounded timeout."""
    import torch.distributed as dist
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist


def allreduce_partials(partial, op: str = "sum"):
    """Combine per-rank partial reductions in place (sum / max / min)."""
    import torch.distributed as dist
    ops = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(partial, op=ops[op])
    return partial


def reduce_leading_axis_sharded(x_shard, out, op: str = "sum"):
    """Sum / max / min over axis 0 of a tensor sharded on axis 0 (CUDA tensors):
    local tadma_b200_reduce over the slab, then one all-reduce of the partial."""
    import tadma_b200 as tb
    from tadma_b200.abi import Reduce
    code = {"sum": Reduce.SUM, "max": Reduce.MAX, "min": Reduce.MIN}[op]
    tb.reduce(code, x_shard, 0, out)
    return allreduce_partials(out, op)


class RankFailure(RuntimeError):
    pass


def run_checked(step, store, rank: int, world: int, tag: str, timeout_s: float = 10.0):
    """Run `step()` on this rank; publish ok/failed in the store and wait (bounded)
    for every rank's verdict before the caller issues its next collective.
    Raises RankFailure on every rank if any rank failed or did not report."""
    import time
    try:
        result = step()
        store.set(f"{tag}/{rank}", "ok")
    except Exception as e:  # the failing rank reports, then re-raises
        store.set(f"{tag}/{rank}", f"failed: {e}")
        raise
    deadline = time.monotonic() + timeout_s
    for r in range(world):
        while True:
            try:
                store.wait([f"{tag}/{r}"], datetime.timedelta(seconds=max(0.01, deadline - time.monotonic())))
                v = store.get(f"{tag}/{r}").decode()
                break
            except Exception:
                raise RankFailure(f"rank {r} did not report step '{tag}' within {timeout_s} s")
        if v != "ok":
            raise RankFailure(f"rank {r} {v}")
    return result
