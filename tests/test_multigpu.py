"""The multi-GPU path on 2 GPUs (one process per GPU, NCCL over NVLink):
row-sharded MLP whose per-rank column sums are combined by the graph's
all_reduce_sum, chunk-sharded chains with no collective, and the failure
paths -- a rank that never joins the communicator, an injected failing
all-reduce on every rank, a rank that leaves between steps (found by the
store heartbeat before the next collective is launched). Nothing here makes
a GPU wait on a peer that will not come: every failure is seen on the host.
NVLS is off (NCCL_NVLS_ENABLE=0)."""
import datetime
import multiprocessing as mp
import os
import socket
import time
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def gpu_count():
    import torch

    return torch.cuda.device_count()


needs2 = pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(target, world=2, timeout=180, extra_env=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q, extra_env or {})) for r in range(world)]
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
    q.put((rank, val))
    q.close()
    q.join_thread()


def setup(rank, world, port, env):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "TT_LAZY_DEVICE": str(rank),
                       "NCCL_NVLS_ENABLE": "0"})
    os.environ.update(env)
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import tt_lazy_b200 as tl

    tl.backend_init()
    return tl, dist


def mlp_inputs():
    rng = np.random.default_rng(21)
    X = rng.standard_normal((512, 256)).astype(np.float32)
    W1 = (rng.standard_normal((256, 512)) / 16).astype(np.float32)
    W2 = (rng.standard_normal((512, 128)) / np.sqrt(512)).astype(np.float32)
    return X, W1, W2


def _mlp_worker(rank, world, port, q, env):
    try:
        tl, dist = setup(rank, world, port, env)
        from tt_lazy_b200 import shard

        shard.init_comm(world, rank, 30000)
        tl.set_gemm_path("ffma")
        X, W1, W2 = mlp_inputs()
        a, b = shard.row_range(X.shape[0], world, rank)
        y = tl.sigmoid(tl.matmul(tl.relu(tl.matmul(tl.constant(np.ascontiguousarray(X[a:b])), tl.constant(W1))),
                                 tl.constant(W2)))
        s = tl.all_reduce_sum(tl.reduce_sum(y, [0]))
        out = s.numpy().copy()
        tl.comm_destroy()
        dist.destroy_process_group()
        post(q, rank, out)
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def _chunk_worker(rank, world, port, q, env):
    try:
        tl, dist = setup(rank, world, port, env)
        from tt_lazy_b200 import shard

        rng = np.random.default_rng(22)
        A = rng.uniform(-1, 1, (512, 256)).astype(np.float32)
        mine = shard.owned_chunks(8, world, rank)
        rows = A[mine[0] * 64:(mine[-1] + 1) * 64]  # the row block of A this rank's chunks read
        T = tl.transpose(tl.constant(np.ascontiguousarray(rows)))
        outs = [tl.reduce_sum(tl.multiply(tl.sigmoid(ch), tl.relu(tl.add(ch, ch))), [1]) for ch in tl.split(T, 64, 1)]
        tl.evaluate(outs)
        post(q, rank, {c: o.numpy().copy() for c, o in zip(mine, outs)})
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def _never_joins_worker(rank, world, port, q, env):
    try:
        tl, dist = setup(rank, world, port, env)
        uid = tl.comm_unique_id() if rank == 0 else None
        obj = [uid]
        dist.broadcast_object_list(obj, src=0)
        if rank == 1:
            post(q, rank, "stayed out")
            os._exit(0)
        t0 = time.monotonic()
        try:
            tl.comm_init(world, rank, obj[0], 3000)
            post(q, rank, "no error")
        except RuntimeError as e:
            post(q, rank, ("error", time.monotonic() - t0, str(e)))
        os._exit(0)
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def _injected_fault_worker(rank, world, port, q, env):
    try:
        tl, dist = setup(rank, world, port, env)
        from tt_lazy_b200 import shard

        shard.init_comm(world, rank, 30000)
        os.environ["TTC_COMM_FAULT"] = "allreduce"  # every rank: nobody launches the collective
        s = tl.all_reduce_sum(tl.reduce_sum(tl.relu(tl.constant(np.ones((4, 8), np.float32))), [0]))
        try:
            s.numpy()
            post(q, rank, "no error")
        except RuntimeError as e:
            post(q, rank, ("error", str(e)))
        os.environ.pop("TTC_COMM_FAULT")
        tl.comm_destroy()
        os._exit(0)
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


def _leaves_between_steps_worker(rank, world, port, q, env):
    try:
        tl, dist = setup(rank, world, port, env)
        from torch.distributed import distributed_c10d as c10d

        from tt_lazy_b200 import shard

        shard.init_comm(world, rank, 30000)
        hb = shard.Heartbeat(c10d._get_default_store(), world, rank, timeout_s=3.0)
        x = np.full((4, 8), rank + 1, np.float32)
        hb.beat(0)
        first = tl.all_reduce_sum(tl.reduce_sum(tl.constant(x), [0])).numpy().copy()  # step 0: 1 + 2 per column x 4
        tl.synchronize()
        if rank == 1:
            post(q, rank, "left")
            os._exit(0)  # between steps: its collective completed, nothing in flight
        t0 = time.monotonic()
        try:
            hb.beat(1)  # step 1 is never launched: the peer is gone
            post(q, rank, "no error")
        except shard.PeerLost as e:
            post(q, rank, ("PeerLost", time.monotonic() - t0, float(first[0]), str(e)))
        os._exit(0)
    except Exception:  # noqa: BLE001
        post(q, rank, traceback.format_exc())


@needs2
def test_row_sharded_mlp_all_reduce_matches_the_full_batch():
    import oracle

    res = run_ranks(_mlp_worker)
    assert sorted(res) == [0, 1], res
    X, W1, W2 = mlp_inputs()
    y = oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X, W1)), W2))
    want = oracle.reduce(y, (0,), f64=True)
    for r in (0, 1):
        assert isinstance(res[r], np.ndarray), res[r]
        assert np.allclose(res[r], want, rtol=1e-5, atol=1e-5)
        assert np.array_equal(res[0], res[r])  # every rank holds the same sum


@needs2
def test_chunk_sharded_chains_without_a_collective():
    import oracle

    res = run_ranks(_chunk_worker)
    assert sorted(res) == [0, 1], res
    rng = np.random.default_rng(22)
    A = rng.uniform(-1, 1, (512, 256)).astype(np.float32)
    t = oracle.transpose(A)
    got = {}
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
        got.update(res[r])
    assert sorted(got) == list(range(8))
    for c in range(8):
        ch = np.ascontiguousarray(t[:, 64 * c:64 * (c + 1)])
        y = oracle.multiply(oracle.sigmoid(ch), oracle.relu(oracle.add(ch, ch)))
        assert np.allclose(got[c], oracle.reduce(y, (1,), f64=True), rtol=1e-5, atol=1e-6)


@needs2
def test_rank_that_never_joins_times_out_communicator_init():
    res = run_ranks(_never_joins_worker)
    assert res.get(1) == "stayed out", res
    kind, waited, msg = res[0]
    assert kind == "error" and ("within" in msg or "failed" in msg), msg
    assert waited < 30.0


@needs2
def test_injected_all_reduce_fault_raises_on_every_rank():
    res = run_ranks(_injected_fault_worker)
    for r in (0, 1):
        assert isinstance(res.get(r), tuple), res
        assert res[r][0] == "error" and "injected" in res[r][1]


@needs2
def test_rank_leaving_between_steps_is_found_before_the_next_collective():
    res = run_ranks(_leaves_between_steps_worker)
    assert res.get(1) == "left", res
    kind, waited, first, msg = res[0]
    assert first == 12.0  # step 0 all-reduced: (1 + 2) * 4 rows
    assert kind == "PeerLost" and "[1]" in msg and waited < 20.0
