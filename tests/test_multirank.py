"""Host logic of the multi-GPU path, on CPU ranks (gloo, world size 2):
row sharding of the batch, the per-rank partial reduction combined by one
all-reduce, and failure detection -- a rank that leaves between steps is
found by the store heartbeat before the next collective, and a collective
whose peer died ends with an error within the process-group timeout instead
of hanging."""
import datetime
import multiprocessing as mp
import os
import socket
import time
import traceback

import numpy as np
import pytest

from tt_lazy_b200 import shard


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(target, world=2, timeout=120, args=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + tuple(args)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.monotonic() + timeout
    while len(results) < world and time.monotonic() < deadline:
        try:
            r, val = q.get(timeout=max(0.1, deadline - time.monotonic()))
            results[r] = val
        except Exception:  # noqa: BLE001 - queue.Empty
            break
    for p in procs:
        p.join(timeout=max(1.0, deadline - time.monotonic()))
        if p.is_alive():
            p.kill()
            p.join()
    return results


def post(q, rank, val):
    """Queue a worker's one result and flush it (the worker may _exit next)."""
    q.put((rank, val))
    q.close()
    q.join_thread()


def init_pg(rank, world, port, seconds):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=seconds))
    return dist


def mlp_inputs():
    rng = np.random.default_rng(11)
    X = rng.standard_normal((66, 32)).astype(np.float32)  # 66 rows: shards of 33 + 33
    W1 = (rng.standard_normal((32, 48)) / np.sqrt(32)).astype(np.float32)
    W2 = (rng.standard_normal((48, 16)) / np.sqrt(48)).astype(np.float32)
    return X, W1, W2


def column_sums(X, W1, W2):
    import oracle

    y = oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X, W1)), W2))
    return oracle.reduce(y, (0,), f64=True).astype(np.float32)


def _sharded_worker(rank, world, port, q):
    try:
        import torch

        dist = init_pg(rank, world, port, 30)
        X, W1, W2 = mlp_inputs()
        a, b = shard.row_range(X.shape[0], world, rank)
        part = torch.from_numpy(column_sums(X[a:b], W1, W2))
        dist.all_reduce(part)
        post(q, rank, part.numpy())
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def _heartbeat_worker(rank, world, port, q):
    try:
        dist = init_pg(rank, world, port, 30)
        from torch.distributed import distributed_c10d as c10d

        hb = shard.Heartbeat(c10d._get_default_store(), world, rank, timeout_s=2.0)
        hb.beat(0)
        if rank == 1:
            post(q, rank, "left")
            os._exit(0)  # leaves between steps, with nothing in flight
        t0 = time.monotonic()
        try:
            hb.beat(1)
            post(q, rank, "no error")
        except shard.PeerLost as e:
            post(q, rank, ("PeerLost", time.monotonic() - t0, str(e)))
        os._exit(0)
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def _dead_peer_worker(rank, world, port, q):
    try:
        import torch

        dist = init_pg(rank, world, port, 5)
        dist.barrier()
        if rank == 1:
            post(q, rank, "failed")
            os._exit(3)  # fails before the collective
        t0 = time.monotonic()
        try:
            dist.all_reduce(torch.ones(4))
            post(q, rank, "no error")
        except Exception as e:  # noqa: BLE001
            post(q, rank, ("error", time.monotonic() - t0, type(e).__name__))
        os._exit(0)
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def test_row_shards_partition_the_batch():
    for rows in (1, 7, 65536, 65537):
        for world in (1, 2, 3, 8):
            spans = [shard.row_range(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == rows
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert [shard.owned_chunks(8, 2, r) for r in range(2)] == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert [shard.owned_chunks(8, 8, r) for r in range(8)] == [[r] for r in range(8)]
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)


def test_sharded_mlp_partial_sums_all_reduce_to_the_full_batch():
    res = run_ranks(_sharded_worker)
    assert sorted(res) == [0, 1], res
    X, W1, W2 = mlp_inputs()
    want = column_sums(X, W1, W2)
    for r in (0, 1):
        assert isinstance(res[r], np.ndarray), res[r]
        assert np.allclose(res[r], want, rtol=1e-5, atol=1e-6)


def test_heartbeat_finds_a_rank_that_left_before_the_next_step():
    res = run_ranks(_heartbeat_worker)
    assert res.get(1) == "left", res
    kind, waited, msg = res[0]
    assert kind == "PeerLost" and "[1]" in msg
    assert waited < 10.0


def test_collective_with_a_dead_peer_errors_within_the_timeout():
    res = run_ranks(_dead_peer_worker)
    assert res.get(1) == "failed", res
    kind, waited, _ = res[0]
    assert kind == "error"
    assert waited < 30.0


def test_cpulist_parsing_and_gpu_numa_lookup(tmp_path):
    """bind_host_to_gpu's topology lookup: the sysfs local_cpulist of the
    GPU's PCI function (a fake sysfs tree here)."""
    from tt_lazy_b200 import shard

    assert shard.parse_cpulist("0-3,8,10-11\n") == [0, 1, 2, 3, 8, 10, 11]
    assert shard.parse_cpulist("") == []
    d = tmp_path / "0000:1b:00.0"
    d.mkdir()
    (d / "local_cpulist").write_text("56-111,168-223\n")
    cpus = shard.gpu_local_cpus((0, 0x1B, 0), str(tmp_path))
    assert cpus[0] == 56 and cpus[-1] == 223 and len(cpus) == 112
    assert shard.gpu_local_cpus((0, 0x1C, 0), str(tmp_path)) is None
    (d / "local_cpulist").write_text("garbage")
    assert shard.gpu_local_cpus((0, 0x1B, 0), str(tmp_path)) is None
