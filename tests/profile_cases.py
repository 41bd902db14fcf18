"""Small, self-contained launches of the hot kernels for profiling (the
cases the ncu summaries under profiles/ were captured on; not a test module).

    python tests/profile_cases.py gemm [M] [tf32|tf32x3|ffma]  # the GEMM path's kernel: X[M,4096] . W[4096,16384], 3 launches
    python tests/profile_cases.py chain NAME [N] # one chain kernel on an N x N fp32 input, 3 launches
    python tests/profile_cases.py small_mlp      # the small MLP workload through tl.Plan, 3 runs
    python tests/profile_cases.py transpose [N]  # transpose_kernel on an N x N fp32 input, 3 launches

NAME: copy | readme (relu -> add -> multiply, stored, summed) | sigmoid |
segments (sigmoid(C) * relu(C + C) over 8 row segments, column sums).
Inputs are seeded, device-resident and larger than L2 at the default sizes;
nothing is timed here (profile with ncu, time with bench.py).
"""
from __future__ import annotations

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _setup():
    import torch

    from tt_lazy_b200 import capi as ttc

    ttc.init(0)
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    ttc.check(ttc.lib().ttc_set_stream(ttc.C.c_void_p(s.cuda_stream)))
    return torch, ttc


def gemm(M=8192, N=16384, K=4096, reps=3, path="tf32"):
    torch, ttc = _setup()
    g = torch.Generator(device="cuda").manual_seed(2)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(K, N, device="cuda", generator=g) / 64
    c = torch.empty(M, N, device="cuda")
    for _ in range(reps):
        ttc.gemm(M, N, K, a.data_ptr(), K, b.data_ptr(), N, c.data_ptr(), N,
                 path={"tf32x3": ttc.GEMM_TF32X3, "ffma": ttc.GEMM_FFMA}.get(path, ttc.GEMM_TF32))
    torch.cuda.synchronize()
    print(f"gemm {path} {M}x{N}x{K} ok, c[0,0] = {float(c[0, 0]):.6g}")


def chain(name="segments", N=8192, reps=3):
    torch, ttc = _setup()
    I = ttc.instr
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.rand(N, N, device="cuda", generator=g) * 2 - 1
    w = torch.empty_like(x)
    s = torch.empty(8, N, device="cuda")
    if name == "segments":
        prog = [I(ttc.OP_LOAD, idx=0), I(ttc.OP_ADD, ttc.SRC_ACC), I(ttc.OP_RELU), I(ttc.OP_SAVE, idx=0),
                I(ttc.OP_LOAD, idx=0), I(ttc.OP_SIGMOID), I(ttc.OP_MUL, ttc.SRC_SLOT, 0)]
        d = ttc.chain_desc(N // 8, N, [ttc.in_view(x.data_ptr(), N, 1, N * N // 8)], [], prog,
                           reduce=ttc.REDUCE_COLS, reduce_out=s.data_ptr(), nseg=8, reduce_seg_stride=N)
    else:
        progs = {
            "copy": ([I(ttc.OP_LOAD, idx=0), I(ttc.OP_STORE, idx=0)], ttc.REDUCE_NONE),
            "readme": ([I(ttc.OP_LOAD, idx=0), I(ttc.OP_RELU), I(ttc.OP_ADD, ttc.SRC_ACC), I(ttc.OP_MUL, ttc.SRC_ACC),
                        I(ttc.OP_STORE, idx=0)], ttc.REDUCE_ALL),
            "sigmoid": ([I(ttc.OP_LOAD, idx=0), I(ttc.OP_SIGMOID), I(ttc.OP_STORE, idx=0)], ttc.REDUCE_NONE),
        }
        prog, red = progs[name]
        d = ttc.chain_desc(N, N, [ttc.in_view(x.data_ptr(), N)], [ttc.out_view(w.data_ptr(), N)], prog, reduce=red,
                           reduce_out=s.data_ptr())
    for _ in range(reps):
        ttc.eltwise_chain(d)
    torch.cuda.synchronize()
    print(f"chain {name} {N}x{N} ok")


def transpose(N=8192, reps=3):
    torch, ttc = _setup()
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.rand(N, N, device="cuda", generator=g)
    y = torch.empty_like(x)
    for _ in range(reps):
        ttc.transpose(x.data_ptr(), y.data_ptr(), 1, N, N)
    torch.cuda.synchronize()
    assert bool((y[:64, :64] == x[:64, :64].T).all())
    print(f"transpose {N}x{N} ok")


def small_mlp(reps=3):
    import torch

    import tt_lazy_b200 as tl
    from tt_lazy_b200 import workloads

    tl.backend_init()
    m, _ = workloads.small_mlp()
    plan = tl.Plan([m])
    for _ in range(reps):
        plan.run()
    torch.cuda.synchronize()
    print(f"small_mlp ok, m[0] = {float(plan.numpy(0)[0]):.6g}, {plan.kernels_last_run} kernels per run")


def main(argv):
    if len(argv) >= 2 and argv[1] == "small_mlp":
        small_mlp()
        return 0
    if len(argv) >= 2 and argv[1] == "transpose":
        transpose(int(argv[2]) if len(argv) > 2 else 8192)
        return 0
    if len(argv) < 2 or argv[1] not in ("gemm", "chain"):
        print(__doc__)
        return 2
    if argv[1] == "gemm":
        gemm(int(argv[2]) if len(argv) > 2 else 8192, path=argv[3] if len(argv) > 3 else "tf32")
    else:
        chain(argv[2] if len(argv) > 2 else "segments", int(argv[3]) if len(argv) > 3 else 8192)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
