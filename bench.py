"""Benchmark of the tt_lazy B200 backend on its headline workloads.

Headline (metric "fused-MLP TFLOP/s"): the large fp32 MLP, batch-sharded over
the GPUs of one node -- X[65536, 4096] ~ N(0,1), W1[4096, 16384] and
W2[16384, 4096] ~ N(0, 1/fan_in) (seed 2, synthetic), Y = sigmoid(relu(X W1)
W2), s = reduce_sum(Y, dim 0) all-reduced across ranks. One step is one
evaluation of that graph through the public front end (a compiled tape:
two tcgen05 TF32 GEMMs with fused relu / sigmoid epilogues, the column
reduction, the NCCL all-reduce when N > 1). The global batch is fixed (strong
scaling); each rank holds 65536/N rows and a full copy of the weights.

Beside it, in the same JSON line: the bandwidth graph (A[16384, 16384] ~
U(-1,1), seed 3: transpose -> 8 column chunks -> sigmoid(C) * relu(C + C) ->
reduce_sum dim 1) as "eltwise_chain" in HBM GB/s, the roofline of the
dominant kernel, a CPU baseline (the reference's own code, compiled from its
sources, on a row sample), the end-to-end number through the public API with
host buffers, and the SM clocks seen while timing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_GLOBAL, K1, N1 = 65536, 4096, 16384
FLOP_STEP = 2 * M_GLOBAL * K1 * N1 * 2  # two GEMMs: 1.759e13
CHAIN_N, CHAIN_SPLIT = 16384, 2048
CHAIN_BYTES = CHAIN_N * CHAIN_N * 4 + 8 * CHAIN_N * 4


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class Clocks:
    """SM clock and throttle-reason samples of this process's GPU taken while
    the timed region runs: NVML read every 2 ms from a background thread (the
    GPU is found by its PCI bus id, so CUDA_VISIBLE_DEVICES does not matter).
    Only reads; changes nothing."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device):
        self.device = device
        self.samples, self.max_mhz, self.reasons = [], None, set()
        self.error = None

    def __enter__(self):
        self.stop = threading.Event()
        self.thread = None
        try:
            import pynvml as nv
            import torch

            nv.nvmlInit()
            try:
                p = torch.cuda.get_device_properties(self.device)
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:  # noqa: BLE001 - no PCI ids: NVML index of the visible device
                vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
                ids = [v for v in vis.split(",") if v.strip().isdigit()]
                self.h = nv.nvmlDeviceGetHandleByIndex(int(ids[self.device]) if ids else self.device)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.nv = nv
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception as e:  # noqa: BLE001
            self.error = repr(e)
        return self

    def _poll(self):
        nv = self.nv
        while not self.stop.is_set():
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, const in self.REASONS:
                    if bits & getattr(nv, const):
                        self.reasons.add(name)
            except Exception as e:  # noqa: BLE001
                self.error = repr(e)
                return
            time.sleep(0.002)

    def __exit__(self, *exc):
        self.stop.set()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "error": self.error}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml, 2 ms"}


# ------------------------------------------------------------------ helpers
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def pinned(shape, capi):
    """numpy view of pinned host memory (fast H2D for the end-to-end run)."""
    n = int(np.prod(shape))
    p = C.c_void_p()
    capi.check(capi.lib().ttc_host_alloc(n * 4, C.byref(p)))
    buf = (C.c_float * n).from_address(p.value)
    return np.ctypeslib.as_array(buf).reshape(shape), p.value


X_BLOCK = 8192  # X is generated in seeded row blocks, so a shard is the same rows at every world size


def _shard_module():
    """tt_lazy_b200/shard.py loaded by path: its row and chunk partition
    (pure Python) without importing the package, whose __init__ loads the
    backend's shared libraries -- the reference arm must not map those."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("tt_lazy_shard_partition",
                                                  os.path.join(ROOT, "tt_lazy_b200", "shard.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def workload_config(world):
    """The `config` of both arms' JSON lines (identical for the same N)."""
    return {"workload": "large fp32 MLP X[65536,4096] W1[4096,16384] W2[16384,4096] relu->sigmoid, "
                        "reduce_sum over batch (all-reduced across ranks); seed 2",
            "global_batch": M_GLOBAL, "parallelism": f"dp{world} (batch-sharded)",
            "l2": "inputs larger than L2 (X shard >= 128 MiB, W1/W2 256 MiB)"}


def make_inputs(rank, world):
    rng = np.random.default_rng(2)
    W1 = (rng.standard_normal((K1, N1), dtype=np.float32) / np.float32(np.sqrt(K1)))
    W2 = (rng.standard_normal((N1, K1), dtype=np.float32) / np.float32(np.sqrt(N1)))
    a, b = _shard_module().row_range(M_GLOBAL, world, rank)
    X = np.empty((b - a, K1), np.float32)
    for blk in range(a // X_BLOCK, (b + X_BLOCK - 1) // X_BLOCK):
        rows = np.random.default_rng(2000 + blk).standard_normal((X_BLOCK, K1), dtype=np.float32)
        lo, hi = max(a, blk * X_BLOCK), min(b, (blk + 1) * X_BLOCK)
        X[lo - a:hi - a] = rows[lo - blk * X_BLOCK:hi - blk * X_BLOCK]
    return X, W1, W2


def chain_rows(chunks):
    """Rows of A[16384, 16384] ~ U(-1,1) that split chunks `chunks` of
    transpose(A) read (chunk i = rows 2048 i .. 2048 i + 2047), each chunk's
    rows from its own seeded stream (seed 3)."""
    out = np.empty((len(chunks) * CHAIN_SPLIT, CHAIN_N), np.float32)
    for j, c in enumerate(chunks):
        out[j * CHAIN_SPLIT:(j + 1) * CHAIN_SPLIT] = np.random.default_rng(3000 + c).uniform(
            -1, 1, (CHAIN_SPLIT, CHAIN_N)).astype(np.float32)
    return out


# ------------------------------------------------------------- CPU baseline
def cpu_reference_rate(X, W1, W2, threads, seconds_target=12.0, rows_per_call=8):
    """TFLOP/s of the reference's own CPU code (oracle/_ref) on a row sample."""
    import oracle

    R = oracle.Ref()
    L = R.L
    w1s = np.asarray(W1.shape, np.uint32)
    w2s = np.asarray(W2.shape, np.uint32)
    rc = L.ref_mlp_prepare(W1.ctypes.data_as(C.c_void_p), w1s.ctypes.data_as(C.c_void_p),
                           W2.ctypes.data_as(C.c_void_p), w2s.ctypes.data_as(C.c_void_p))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    flop_row = 2 * K1 * N1 * 2
    done = [0] * threads
    stop = time.perf_counter() + seconds_target

    def work(t):
        out = np.empty(K1, np.float32)
        r0 = (t * rows_per_call * 97) % (X.shape[0] - rows_per_call)
        while time.perf_counter() < stop:
            xs = np.ascontiguousarray(X[r0:r0 + rows_per_call])
            rc = L.ref_mlp_rows(xs.ctypes.data_as(C.c_void_p), C.c_uint32(rows_per_call), C.c_uint32(K1),
                                out.ctypes.data_as(C.c_void_p))
            if rc != 0:
                raise RuntimeError(L.ref_last_error().decode())
            done[t] += rows_per_call
            r0 = (r0 + rows_per_call * threads) % (X.shape[0] - rows_per_call)

    t0 = time.perf_counter()
    ths = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    dt = time.perf_counter() - t0
    rows = sum(done)
    return rows * flop_row / dt / 1e12, rows, dt


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    import oracle

    if oracle.ref() is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libttref.so was not built"}))
        return
    X, W1, W2 = make_inputs(0, 1)
    threads = os.cpu_count() or 1
    vals = []
    for i in range(args.warmup + args.steps):
        v, rows, dt = cpu_reference_rate(X, W1, W2, threads, seconds_target=args.ref_seconds)
        if i >= args.warmup:
            vals.append((v, rows, dt))
    v = statistics.median([x[0] for x in vals])
    sample = f"{vals[-1][1]} rows of X per step ({threads} threads x 8-row calls, ~{args.ref_seconds:.0f} s), " \
             f"extrapolated to the full 65536-row step"
    line = {
        "metric": "fused-MLP TFLOP/s", "value": v, "unit": "TFLOP/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": FLOP_STEP / (v * 1e12) * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) inputs, N(0,1/fan_in) weights)",
        "config": workload_config(world),
        "arm": {"runs_on": f"host CPU, {threads} threads (rank 0 only)",
                "code": "the reference's math::matmul / math::relu compiled from its sources (oracle/_ref)"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def _device_ms(torch, stream, fn, reps):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def other_configs(torch, tl, stream, hbm_peak, tf32_peak):
    """README chain (1000^2 as configured, and 16384^2 for the HBM figure),
    the small MLP and the DAG stress graph, each through tl.Plan; the small
    ones also as captured CUDA graphs (launch-bound at their sizes)."""
    from tt_lazy_b200 import workloads

    out, launches = {}, 0

    def plan_times(outs, reps, capture=True):
        nonlocal launches
        plan = tl.Plan(outs)
        for _ in range(3):
            plan.run()
        ms = _device_ms(torch, stream, plan.run, reps)
        launches += plan.kernels_last_run * (reps + 3)
        res = {"ms": ms, "kernels_per_run": plan.kernels_last_run, "tape_ops": len(plan)}
        if capture:
            plan.capture()
            for _ in range(3):
                plan.run()
            res["ms_graph"] = _device_ms(torch, stream, plan.run, reps)
            launches += plan.kernels_last_run * (reps + 3)
        return plan, res

    # README chain
    w, s, work = workloads.readme_chain(1000)
    plan, r = plan_times([w, s], 200)
    out["readme_chain_1000"] = {
        "workload": "x[1000,1000] U(-1,1) seed 0: w = (relu(x) + relu(x))^2, s = sum(w); outputs w and s",
        "bytes": work["bytes"], "us_per_run": r["ms"] * 1e3, "us_per_run_graph": r["ms_graph"] * 1e3,
        "GBs_graph": work["bytes"] / (r["ms_graph"] * 1e-3) / 1e9, "kernels_per_run": r["kernels_per_run"],
        "note": "8 MB fits in L2: launch-bound"}
    del plan, w, s
    w, s, work = workloads.readme_chain(16384)
    plan, r = plan_times([w, s], 20, capture=False)
    gbs = work["bytes"] / (r["ms"] * 1e-3) / 1e9
    out["readme_chain_16384"] = {
        "workload": "the same chain on x[16384,16384] (2 GiB moved per run)", "bytes": work["bytes"],
        "ms_per_run": r["ms"], "GBs": gbs, "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm_peak,
                                                        "unit": "GB/s", "frac": gbs / hbm_peak},
        "kernels_per_run": r["kernels_per_run"]}
    del plan, w, s
    tl.clear_cache()
    # small MLP
    m, work = workloads.small_mlp()
    plan, r = plan_times([m], 200)
    out["small_mlp"] = {
        "workload": "X[256,512] N(0,1), W1[512,1024], W2[1024,512] N(0,1/fan_in), b U(-0.1,0.1), seed 1: "
                    "reduce_mean(relu(X W1 + b1) W2 + b2, dim 0)",
        "flops": work["flops"], "us_per_run": r["ms"] * 1e3, "us_per_run_graph": r["ms_graph"] * 1e3,
        "TFLOPs_graph": work["flops"] / (r["ms_graph"] * 1e-3) / 1e12, "kernels_per_run": r["kernels_per_run"],
        "tape_ops": r["tape_ops"], "note": "0.5 GFLOP: launch- and latency-bound"}
    del plan, m
    tl.clear_cache()
    # DAG stress: the seeded inputs and topology are drawn first; the clock
    # covers creating the graph nodes (constants included) only
    inputs, program, work = workloads.dag_stress_program()
    t0 = time.perf_counter()
    outs = workloads.dag_build(inputs, program, work["sinks"])
    t1 = time.perf_counter()
    plan = tl.Plan(outs)
    t2 = time.perf_counter()
    plan.run()
    torch.cuda.synchronize()
    t3 = time.perf_counter()
    for _ in range(2):
        plan.run()
    ms = _device_ms(torch, stream, plan.run, 5)
    launches += plan.kernels_last_run * 8
    out["dag_stress"] = {
        "workload": f"random DAG seed 4: {work['graph_nodes']} nodes over [4096,4096] "
                    f"({work['dead_ops']} unreachable), ops {work['counts']}, reduce_sum(dim 1) at 4 sinks",
        "graph_build_ms": (t1 - t0) * 1e3, "tape_build_ms": (t2 - t1) * 1e3,
        "first_eval_ms": (t3 - t2) * 1e3,
        "note": "graph_build_ms: creating the 204 graph nodes and 5 constants (inputs drawn before the clock); "
                "tape_build_ms: tape generation, DCE and fusion passes; first_eval_ms includes compiling the "
                "program-specialised chain kernels (NVRTC, once per program)",
        "eval_ms": ms, "tape_ops": len(plan), "kernels_per_run": plan.kernels_last_run,
        "live_ops": work["live_ops"], "flops": work["flops"], "bytes_unfused": work["bytes_unfused"],
        "TFLOPs": work["flops"] / (ms * 1e-3) / 1e12,
        "matmul_roofline_frac": (work["flops"] / (ms * 1e-3) / 1e12) / tf32_peak}
    del plan, outs, inputs
    tl.clear_cache()
    out["_launches"] = launches
    return out


def run_ours(args):
    import torch

    world, rank, local = dist_env()
    os.environ.setdefault("TT_LAZY_DEVICE", str(local))
    torch.cuda.set_device(local)
    import tt_lazy_b200 as tl
    from tt_lazy_b200 import capi
    from tt_lazy_b200 import shard as _shard

    # host staging buffers on the GPU's own socket (allocated after this)
    numa_cpus = _shard.bind_host_to_gpu(local) if world > 1 else None

    tl.backend_init()
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        from tt_lazy_b200 import shard

        shard.init_comm(world, rank, 60000)
    stream = torch.cuda.ExternalStream(tl.stream())

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    X, W1, W2 = make_inputs(rank, world)
    rows = X.shape[0]

    def graph(xt):
        h = tl.relu(tl.matmul(xt, tl.constant(W1)))
        y = tl.sigmoid(tl.matmul(h, tl.constant(W2)))
        s = tl.reduce_sum(y, [0])
        return tl.all_reduce_sum(s) if world > 1 else s

    # ---- device-resident inputs: the hot path alone. The batch runs as row
    # chunks of 8192 (constant row views of the resident X, the same work):
    # under the 1 kW cap the shorter GEMM pairs hold higher clocks (measured
    # alternately: 553-572 TFLOP/s in 8 chunks vs 477-513 as one batch).
    s_dev = graph(tl.constant(X))
    res_chunks = max(1, rows // 8192)
    plan = tl.Plan([s_dev], pipeline_chunks=res_chunks) if res_chunks > 1 else tl.Plan([s_dev])
    for _ in range(args.warmup):
        plan.run()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            plan.run()
        e1.record(stream)
        barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    launches = plan.kernels_last_run * args.steps
    value = FLOP_STEP / (ms * 1e-3) / 1e12
    s_val = plan.numpy(0)
    assert np.all(np.isfinite(s_val)), "non-finite result"

    # ---- end to end through the public API with host buffers
    Xp, _ = pinned(X.shape, capi)
    Xp[...] = X
    s_e2e = graph(tl.streamed(Xp))
    # row-chunked plan: chunk c + 1 uploads on the copy stream while chunk c computes
    chunks = max(1, min(8, rows // 2048))
    plan_e2e = tl.Plan([s_e2e], pipeline_chunks=chunks) if chunks > 1 else tl.Plan([s_e2e])
    for _ in range(max(1, args.warmup - 1)):
        plan_e2e.run()
        plan_e2e.numpy(0)
    barrier()
    t0 = time.perf_counter()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        plan_e2e.run()
        out = plan_e2e.numpy(0)  # the device -> host read of the step's result
    e3.record(stream)
    barrier()
    ms_e2e = max_over_ranks(max(e2.elapsed_time(e3), (time.perf_counter() - t0) * 1e3) / args.steps)
    e2e_value = FLOP_STEP / (ms_e2e * 1e-3) / 1e12
    del plan_e2e, s_e2e

    # ---- roofline of the dominant kernel: the first GEMM (TF32 tcgen05) timed alone
    hbm_peak, bf16_peak, peak_kind = peaks()
    tf32_peak = bf16_peak / 2.0
    Xd = capi.DeviceArray.from_numpy(X[: min(rows, 16384)])
    W1d = capi.DeviceArray.from_numpy(W1)
    Hd = capi.DeviceArray.empty((Xd.shape[0], N1))
    capi.check(capi.lib().ttc_set_stream(C.c_void_p(tl.stream())))
    Mg = Xd.shape[0]

    def one_gemm():
        capi.gemm(Mg, N1, K1, Xd.ptr, K1, W1d.ptr, N1, Hd.ptr, N1, path=capi.GEMM_TF32)

    for _ in range(3):
        one_gemm()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    reps = 10
    for _ in range(reps):
        one_gemm()
    g1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = g0.elapsed_time(g1) / reps
    gemm_tflops = 2 * Mg * N1 * K1 / (gemm_ms * 1e-3) / 1e12
    launches += reps + 3
    # The library's default picks the CTA-pair kernel (tcgen05.mma.cta_group::2)
    # when its 256x256 tiles fill the GPU (at least one per CTA pair); the other
    # kernel is timed on the same GEMM for comparison.
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    pair_default = Mg >= 256 and N1 >= 256 and ((Mg + 255) // 256) * ((N1 + 255) // 256) >= sms // 2
    os.environ["TTC_GEMM_PAIR"] = "0" if pair_default else "1"
    for _ in range(3):
        one_gemm()
    torch.cuda.synchronize()
    g0.record(stream)
    for _ in range(reps):
        one_gemm()
    g1.record(stream)
    torch.cuda.synchronize()
    os.environ.pop("TTC_GEMM_PAIR")
    alt_ms = g0.elapsed_time(g1) / reps
    launches += reps + 3
    # the fp32-accurate three-pass TF32 path on the same GEMM (operand split + 3 MMAs per step)
    for _ in range(3):
        capi.gemm(Mg, N1, K1, Xd.ptr, K1, W1d.ptr, N1, Hd.ptr, N1, path=capi.GEMM_TF32X3)
    torch.cuda.synchronize()
    g0.record(stream)
    for _ in range(reps):
        capi.gemm(Mg, N1, K1, Xd.ptr, K1, W1d.ptr, N1, Hd.ptr, N1, path=capi.GEMM_TF32X3)
    g1.record(stream)
    torch.cuda.synchronize()
    x3_ms = g0.elapsed_time(g1) / reps
    launches += 3 * (reps + 3)
    traffic = None
    tp = os.path.join(ROOT, "profiles", "tf32_gemm_traffic.txt")
    if os.path.exists(tp):
        try:
            key = "bytes_per_flop_pair=" if pair_default else "bytes_per_flop="
            per_flop = float(open(tp).read().split(key)[1].split()[0])
            traffic = per_flop * 2 * Mg * N1 * K1
        except Exception:
            traffic = None
    del Xd, W1d, Hd

    # ---- bandwidth graph (eltwise chain block): chunk i of the split on the
    # rank that owns it, which holds only the rows of A its chunks read; no
    # collective (strong scaling over the 8 chunks)
    chain = None
    if not args.skip_chain:
        from tt_lazy_b200 import shard

        mine = shard.owned_chunks(CHAIN_N // CHAIN_SPLIT, world, rank)
        A = chain_rows(mine)
        T = tl.transpose(tl.constant(A))
        outs = [tl.reduce_sum(tl.multiply(tl.sigmoid(ch), tl.relu(tl.add(ch, ch))), [1])
                for ch in tl.split(T, CHAIN_SPLIT, 1)]
        cplan = tl.Plan(outs)
        cplan.capture()  # the chain and its finalize replay as one CUDA graph
        for _ in range(3):
            cplan.run()
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        creps = 20
        c0.record(stream)
        for _ in range(creps):
            cplan.run()
        c1.record(stream)
        barrier()
        cms = max_over_ranks(c0.elapsed_time(c1) / creps)
        gbs = CHAIN_BYTES / (cms * 1e-3) / 1e9  # whole job: all 8 chunks / slowest rank
        per_gpu = gbs / world
        launches += cplan.kernels_last_run * (creps + 3)
        chain = {"metric": "eltwise-chain HBM GB/s", "value": gbs, "unit": "GB/s", "per_gpu": per_gpu,
                 "ms_per_step": cms, "kernels_per_step": cplan.kernels_last_run, "scaling": "strong",
                 "workload": "A[16384,16384] U(-1,1) seed 3: transpose -> 8 column chunks -> "
                             "sigmoid(C)*relu(C+C) -> reduce_sum dim 1; chunks sharded over ranks",
                 "chunks_per_gpu": len(mine), "algorithmic_bytes": CHAIN_BYTES, "launch": "tl.Plan captured as a CUDA graph",
                 "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": hbm_peak, "unit": "GB/s",
                              "frac": per_gpu / hbm_peak, "peak_source": peak_kind}}
        del cplan, outs

    # ---- the other workloads (README chain, small MLP, DAG stress): replicas
    # only, so rank 0 at N = 1 times them
    others = None
    if rank == 0 and world == 1 and not args.skip_configs:
        others = other_configs(torch, tl, stream, hbm_peak, tf32_peak)
        launches += others.pop("_launches")

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        try:
            v, nrows, dt = cpu_reference_rate(X, W1, W2, threads=1, seconds_target=args.ref_seconds)
            cpu = {"value": v, "unit": "TFLOP/s", "cores": 1, "kind": "reference",
                   "sample": f"{nrows} rows of X through the reference's math::matmul/relu in {dt:.1f} s "
                             f"(1 thread of {os.cpu_count()}), extrapolated to 65536 rows"}
        except Exception as e:  # noqa: BLE001
            cpu = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "reference", "sample": f"failed: {e}"}

    if rank == 0:
        clocks = clk.summary()
        kernel_name = {False: "tf32_gemm_kernel (tcgen05, 128x256 tile per CTA)",
                       True: "tf32_gemm_pair_kernel (tcgen05 cta_group::2, 256x256 tile per CTA pair)"}
        line = {
            "metric": "fused-MLP TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 (tf32 tensor-core GEMM, fp32 accumulate)",
            "data": "synthetic (seeded N(0,1) inputs, N(0,1/fan_in) weights)",
            "config": workload_config(world),
            "arm": {"rows_per_gpu": rows, "row_chunks": res_chunks},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": int(X.nbytes), "d2h_bytes_per_step": int(K1 * 4),
                    "host_binding": (f"{len(numa_cpus)} CPUs of the GPU's NUMA node" if numa_cpus else "none"),
                    "path": f"tt_lazy Plan(pipeline_chunks={chunks}).run() over a streamed pinned-host X "
                            "(row chunks uploaded on a copy stream under the previous chunk's GEMMs) "
                            "+ to-host read of s"},
            "roofline": {"bound": "tensor", "kernel": kernel_name[pair_default],
                         "achieved": gemm_tflops, "peak": tf32_peak, "unit": "TFLOP/s",
                         "frac": gemm_tflops / tf32_peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} bf16 dense / 2 (TF32 rate)",
                         "launch_ms": gemm_ms, "shape": [Mg, N1, K1],
                         ("single_cta_kernel" if pair_default else "cta_pair_kernel"): {
                             "kernel": kernel_name[not pair_default],
                             "achieved": 2 * Mg * N1 * K1 / (alt_ms * 1e-3) / 1e12,
                             "launch_ms": alt_ms, "enabled_by": "TTC_GEMM_PAIR=0" if pair_default
                             else "TTC_GEMM_PAIR=1"},
                         "tf32x3_path": {"achieved": 2 * Mg * N1 * K1 / (x3_ms * 1e-3) / 1e12,
                                         "tensor_frac": 3 * 2 * Mg * N1 * K1 / (x3_ms * 1e-3) / 1e12 / tf32_peak,
                                         "ms": x3_ms, "enabled_by": "path TTC_GEMM_TF32X3 (fp32-accurate, 1e-5)",
                                         "note": "fp32 flops per second incl. the operand split; the tensor "
                                                 "cores do 3x the MMA work"}},
            "eltwise_chain": chain,
            "other_configs": others,
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "checksum": float(np.sum(s_val, dtype=np.float64)),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        tl.comm_destroy()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--skip-chain", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-configs", action="store_true")
    ap.add_argument("--ref-seconds", type=float, default=12.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        # keep the whole reference run within a few minutes
        args.ref_seconds = min(args.ref_seconds, 150.0 / (args.steps + args.warmup))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
