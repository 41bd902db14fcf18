"""Randomised differential test of ttc_gemm against the oracle.

Seeded random shapes (ragged and tile-aligned, few output tiles -- split-K --
and many), stored operand layouts (both transposes), paths (FFMA, TF32,
TF32X3) and epilogue programs (bias add from a [1, N] view, an element-wise
product with a full [M, N] operand, relu or sigmoid, up to two stores, and a
fused column sum or mean over the rows). Every stored matrix and the column
sums are compared with the oracle's own steps (the reference's sequential fp32
matmul, then IEEE float32 element-wise steps; sums in fp64) within the path's
norm-wise bound: 1e-5 for FFMA and TF32X3, 2e-3 for TF32.
"""
import ctypes as C

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

TOL = {"ffma": 1e-5, "tf32": 2e-3, "tf32x3": 1e-5, "auto (FFMA for this shape)": 1e-5}


def _normwise(got, want):
    w = want.astype(np.float64)
    return np.linalg.norm(got.astype(np.float64) - w) / max(np.linalg.norm(w), 1e-300)


def _shape(rng, seed):
    if seed % 4 == 3:  # many output tiles: no split-K
        return int(rng.integers(9, 12)) * 128, int(rng.integers(6, 9)) * 256, int(rng.integers(2, 9)) * 32
    m = int(rng.integers(1, 700))
    n = 4 * int(rng.integers(1, 160))
    k = int(rng.integers(1, 900))
    return m, n, k


@pytest.mark.parametrize("seed", range(24))
def test_random_gemm_matches_oracle(ttc, seed):
    rng = np.random.default_rng(2000 + seed)
    m, n, k = _shape(rng, seed)
    ta, tb = int(rng.integers(0, 2)), int(rng.integers(0, 2))
    path = ["ffma", "tf32", "tf32x3"][seed % 3]
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(max(k, 1))).astype(np.float32)
    a_st = np.ascontiguousarray(a.T) if ta else a
    b_st = np.ascontiguousarray(b.T) if tb else b
    A, B = ttc.DeviceArray.from_numpy(a_st), ttc.DeviceArray.from_numpy(b_st)

    bias = rng.uniform(-0.1, 0.1, (1, n)).astype(np.float32)
    gate = rng.uniform(-1, 1, (m, n)).astype(np.float32)
    Bias, Gate = ttc.DeviceArray.from_numpy(bias), ttc.DeviceArray.from_numpy(gate)
    inputs = [ttc.in_view(Bias.ptr, 0), ttc.in_view(Gate.ptr, n)]
    prog, steps = [], []
    if rng.integers(0, 2):
        prog.append(ttc.instr(ttc.OP_ADD, ttc.SRC_INPUT, 0))
        steps.append("bias")
    if rng.integers(0, 3) == 0:
        prog.append(ttc.instr(ttc.OP_MUL, ttc.SRC_INPUT, 1))
        steps.append("gate")
    outs = []
    if rng.integers(0, 2):
        outs.append(ttc.DeviceArray.empty((m, n)))
        prog.append(ttc.instr(ttc.OP_STORE, idx=0))
        steps.append("store")
    act = ["none", "relu", "sigmoid"][int(rng.integers(0, 3))]
    if act != "none":
        prog.append(ttc.instr(ttc.OP_RELU if act == "relu" else ttc.OP_SIGMOID))
        steps.append(act)
    reduce = bool(rng.integers(0, 2))
    mean = bool(rng.integers(0, 2)) and reduce
    if not reduce or rng.integers(0, 2):
        outs.append(ttc.DeviceArray.empty((m, n)))
        prog.append(ttc.instr(ttc.OP_STORE, idx=len(outs) - 1))
        steps.append("store")
    S = ttc.DeviceArray.empty((n,))
    epi = ttc.chain_desc(m, n, inputs, [ttc.out_view(o.ptr, n) for o in outs], prog,
                         reduce=ttc.REDUCE_COLS if reduce else ttc.REDUCE_NONE,
                         reduce_out=S.ptr if reduce else None, mean=mean)
    code = {"ffma": ttc.GEMM_FFMA, "tf32": ttc.GEMM_TF32, "tf32x3": ttc.GEMM_TF32X3}[path]
    g = _desc(ttc, m, n, k, A, a_st.shape[1], B, b_st.shape[1], ta, tb, ttc.GEMM_AUTO, epi)
    if path == "tf32" and ttc.gemm_select_path(g) != ttc.GEMM_TF32:
        path, code = "auto (FFMA for this shape)", ttc.GEMM_AUTO  # the explicit TF32 path rejects it
    g.path = code
    ttc.check(ttc.lib().ttc_gemm(C.byref(g)))

    y = oracle.matmul(a_st, b_st, ta, tb)
    stored = []
    for step in steps:
        if step == "bias":
            y = oracle.add(y, bias)
        elif step == "gate":
            y = oracle.multiply(y, gate)
        elif step == "relu":
            y = oracle.relu(y)
        elif step == "sigmoid":
            y = oracle.sigmoid(y)
        else:
            stored.append(y.copy())
    tol = TOL[path]
    for o, want in zip(outs, stored):
        assert _normwise(o.numpy(), want) <= tol, (path, m, n, k, ta, tb, steps)
    if reduce:
        want = oracle.reduce(y, (0,), mean=mean, f64=True)
        assert _normwise(S.numpy(), want) <= tol, (path, m, n, k, ta, tb, steps, "colsum")


def _desc(ttc, m, n, k, A, lda, B, ldb, ta, tb, path, epi):
    g = ttc.GemmDesc()
    g.M, g.N, g.K = m, n, k
    g.a, g.lda, g.trans_a = A.ptr, lda, ta
    g.b, g.ldb, g.trans_b = B.ptr, ldb, tb
    g.c, g.ldc = None, n
    g.path = path
    g.epilogue = epi
    return g
