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
* ``bind_host_to_gpu(device)`` -- pins the process to the CPUs of the GPU's
  NUMA node (sysfs ``local_cpulist`` of its PCI function), so pinned host
  buffers allocated afterwards are local to the GPU's socket and eight ranks'
  host -> GPU copies do not cross the socket interconnect.
* ``Heartbeat`` -- host-side failure detection between steps: every rank
  checks in on the process group's store before it launches a step's
  collective and raises ``PeerLost`` when a peer has not checked in within
  the deadline, so no rank launches a collective that a lost peer would
  never join.
"""
from __future__ import annotations

import os
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


def parse_cpulist(text: str) -> list[int]:
    """'0-3,8,10-11' -> [0, 1, 2, 3, 8, 10, 11] (the sysfs / cpuset list format)."""
    cpus: list[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        lo, _, hi = part.partition("-")
        cpus.extend(range(int(lo), int(hi or lo) + 1))
    return cpus


def gpu_local_cpus(pci: tuple[int, int, int], sysfs: str = "/sys/bus/pci/devices") -> list[int] | None:
    """CPUs local to the GPU at PCI (domain, bus, device), or None when sysfs
    does not say (no such file, or an empty list)."""
    domain, bus, dev = pci
    path = os.path.join(sysfs, f"{domain:04x}:{bus:02x}:{dev:02x}.0", "local_cpulist")
    try:
        with open(path) as f:
            cpus = parse_cpulist(f.read())
    except (OSError, ValueError):
        return None
    return cpus or None


def bind_host_to_gpu(device: int, sysfs: str = "/sys/bus/pci/devices") -> list[int] | None:
    """Restricts this process to the CPUs of CUDA device `device`'s NUMA node
    (intersected with the CPUs it may already use). Returns the CPUs bound
    to, or None when nothing changed (no topology information, or no
    overlap). Call before allocating pinned host buffers."""
    import torch

    p = torch.cuda.get_device_properties(device)
    cpus = gpu_local_cpus((p.pci_domain_id, p.pci_bus_id, p.pci_device_id), sysfs)
    if not cpus:
        return None
    allowed = os.sched_getaffinity(0)
    use = [c for c in cpus if c in allowed]
    if not use or set(use) == allowed:
        return None
    os.sched_setaffinity(0, use)
    return use


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
