"""Data parallelism of the batch-sharded workloads: one process per GPU.

* ``row_range(rows, world, rank)`` -- the contiguous row block of a batch a
  rank owns (the large MLP is row-separable: each rank runs both GEMMs on its
  rows with replicated weights, and the per-rank column sums are combined by
  one all-reduce, ``all_reduce_sum`` in the graph).
* ``owned_chunks(n, world, rank)`` -- the split chunks a rank evaluates when a
  graph of independent chunks is spread over ranks (no collective).
* ``init_comm(world, rank, timeout_ms)`` -- creates the backend's NCCL
  communicator: rank 0's unique id travels over the already initialised
  ``torch.distributed`` process group (any backend, gloo included).
* ``Heartbeat`` -- host-side failure detection between steps: every rank
  checks in on the process group's store before it launches a step's
  collective and raises ``PeerLost`` when a peer has not checked in within
  the deadline, so no rank launches a collective that a lost peer would
  never join.
"""
from __future__ import annotations

import time


def row_range(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of rank `rank` (blocks differ in size by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def owned_chunks(n_chunks: int, world: int, rank: int) -> list[int]:
    """Chunk indices of rank `rank`: a contiguous block, so that the rows of
    the source a rank needs are contiguous too."""
    start, stop = row_range(n_chunks, world, rank)
    return list(range(start, stop))


def init_comm(world: int, rank: int, timeout_ms: int = 60000) -> None:
    """Creates the backend communicator over the default process group."""
    import torch.distributed as dist

    import tt_lazy_b200 as tl

    uid = tl.comm_unique_id() if rank == 0 else None
    obj = [uid]
    dist.broadcast_object_list(obj, src=0)
    tl.comm_init(world, rank, obj[0], timeout_ms)


class PeerLost(RuntimeError):
    pass


class Heartbeat:
    """Step-level liveness over a ``torch.distributed`` store.

    ``beat(step)`` records this rank at `step` and waits (polling, bounded by
    `timeout_s`) until every rank has recorded `step`; a rank that left or
    failed never does, and the others raise PeerLost instead of launching a
    collective it would never join."""

    def __init__(self, store, world: int, rank: int, timeout_s: float = 10.0, prefix: str = "tt_lazy/hb"):
        self.store, self.world, self.rank = store, world, rank
        self.timeout_s, self.prefix = timeout_s, prefix

    def beat(self, step: int) -> None:
        self.store.set(f"{self.prefix}/{step}/{self.rank}", "1")
        deadline = time.monotonic() + self.timeout_s
        missing = list(range(self.world))
        while True:
            missing = [r for r in missing if not self.store.check([f"{self.prefix}/{step}/{r}"])]
            if not missing:
                return
            if time.monotonic() > deadline:
                raise PeerLost(f"rank(s) {missing} did not reach step {step} within {self.timeout_s:.1f} s")
            time.sleep(0.01)
