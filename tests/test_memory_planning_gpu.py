"""Tape-level memory planning on the device (the HBM MemoryManager that
replaces the reference's unused host pool, src/core/MemoryManager.cpp:46-133
of the reference): a result is released right after its last reader and the
next operation of the same size reuses it, so a chain of same-sized
intermediates needs two live buffers, not one per operation; a captured
plan's buffers return to the pool when the plan goes away."""
import numpy as np
import pytest

import oracle
import tt_lazy_b200 as tl

pytestmark = pytest.mark.gpu

N = 1024
BUF = N * N * 4  # 4 MiB, a multiple of the pool's 2 MiB bucket above 1 MiB


@pytest.fixture(autouse=True)
def fresh():
    tl.clear()
    tl.clear_cache()
    tl.set_gemm_path("ffma")
    yield
    tl.set_gemm_path("auto")
    tl.clear()
    tl.clear_cache()


def _layers(X, W, depth):
    h = tl.constant(X)
    w = tl.constant(W)
    for _ in range(depth):
        h = tl.relu(tl.matmul(h, w))  # one GEMM with a relu epilogue per layer
    return h


def test_chain_of_intermediates_reuses_two_buffers():
    depth = 6
    rng = np.random.default_rng(5)
    X = rng.uniform(-1, 1, (N, N)).astype(np.float32)
    W = (rng.standard_normal((N, N)) / np.sqrt(N)).astype(np.float32)
    out = _layers(X, W, depth)
    s0 = tl.stats()
    tl.reset_peak()
    got = out.numpy()
    s1 = tl.stats()
    # layer i + 1 takes the buffer layer i - 1 released
    assert s1["device_reuses"] - s0["device_reuses"] >= depth - 2, (s0, s1)
    # peak above the start: the two uploaded constants plus two layers live at
    # once (one per layer, 6 x 4 MiB, without liveness release)
    assert s1["device_bytes_peak"] - s0["device_bytes_live"] <= 2 * BUF + 2 * BUF, (s0, s1)
    want = X
    for _ in range(depth):
        want = oracle.relu(oracle.matmul(want, W))
    err = np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))
    assert err <= 1e-5


def test_captured_plan_returns_its_buffers():
    rng = np.random.default_rng(6)
    X = rng.uniform(-1, 1, (N, N)).astype(np.float32)
    W = (rng.standard_normal((N, N)) / np.sqrt(N)).astype(np.float32)
    base = tl.stats()["device_bytes_live"]
    out = _layers(X, W, 4)
    plan = tl.Plan([out])
    plan.capture()
    for _ in range(3):
        plan.run()
    first = plan.numpy(0)
    held = tl.stats()["device_bytes_live"]
    assert held >= base + BUF  # the graph's result (and its claimed intermediates) stay with the plan
    plan.run()
    assert np.array_equal(plan.numpy(0), first)  # replays write the same buffers
    del plan, out
    tl.clear()
    tl.clear_cache()
    assert tl.stats()["device_bytes_live"] == base
