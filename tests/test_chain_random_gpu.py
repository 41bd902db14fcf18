"""Randomised differential test of ttc_eltwise_chain against the oracle.

Seeded random chain programs -- LOAD, RELU, SIGMOID, ADD / MUL with the
accumulator, an input or a saved slot, SAVE, STORE -- over random operand
views (full, row-broadcast [1, C] as in the reference's bias add, column-
broadcast [R, 1]), segment counts and reductions (none, all, rows, columns,
sum or mean), on shapes that reach the register interpreters (small or
ragged: cols not a multiple of 4) and the program-specialised NVRTC kernels
(from 256 Ki elements); the same programs run once more in a fresh process
with the specialised kernels off, where the large layouts take the
TMA-staged interpreter.

Bounds, as in the other parity tests: stored results are bit-exact against
the oracle's IEEE float32 steps, sigmoid included (it returns the
reference formula's float; on a host whose glibc is its build without FMA,
one float of sigmoid is 1 ulp away, and programs with a sigmoid then get a
1e-5 relative bound); reductions are within 1e-5 of the fp64 sum of the
oracle's own element values, relative to the sum of magnitudes.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

SHAPES = [(3, 5), (17, 1028), (64, 100), (256, 256), (1024, 1024), (1200, 1100), (515, 2052)]


def _program(rng, n_inputs):
    """A random program (list of (op, src, idx)) and the ops it uses."""
    prog = [("LOAD", "ACC", 0)]
    saved = []
    n_out = 0
    for _ in range(int(rng.integers(2, 9))):
        k = int(rng.integers(0, 8))
        if k == 0:
            prog.append(("RELU", "ACC", 0))
        elif k == 1:
            prog.append(("SIGMOID", "ACC", 0))
        elif k in (2, 3):
            op = "ADD" if k == 2 else "MUL"
            choice = int(rng.integers(0, 3))
            if choice == 1 and n_inputs > 1:
                prog.append((op, "INPUT", int(rng.integers(1, n_inputs))))
            elif choice == 2 and saved:
                prog.append((op, "SLOT", saved[int(rng.integers(0, len(saved)))]))
            else:
                prog.append((op, "ACC", 0))
        elif k == 4 and len(saved) < 2:
            s = len(saved)
            prog.append(("SAVE", "ACC", s))
            saved.append(s)
        elif k == 5 and n_out < 2:
            prog.append(("STORE", "ACC", n_out))
            n_out += 1
        elif k == 6 and n_inputs > 1:
            prog.append(("LOAD", "ACC", int(rng.integers(0, n_inputs))))
        else:
            prog.append(("RELU", "ACC", 0))
    return prog, n_out


def _evaluate(prog, xs):
    """The oracle's evaluation: every step one IEEE float32 operation."""
    acc = np.zeros_like(xs[0])
    slots, outs = {}, {}
    for op, src, idx in prog:
        if op == "LOAD":
            acc = xs[idx].copy()
        elif op == "RELU":
            acc = oracle.relu(acc)
        elif op == "SIGMOID":
            acc = oracle.sigmoid(acc)
        elif op in ("ADD", "MUL"):
            other = acc if src == "ACC" else xs[idx] if src == "INPUT" else slots[idx]
            acc = (acc + other) if op == "ADD" else (acc * other)
            acc = acc.astype(np.float32)
        elif op == "SAVE":
            slots[idx] = acc.copy()
        elif op == "STORE":
            outs[idx] = acc.copy()
    return acc, outs


@pytest.mark.parametrize("seed", range(40))
def test_random_chain_matches_oracle(ttc, seed):
    rng = np.random.default_rng(1000 + seed)
    rows, cols = SHAPES[seed % len(SHAPES)]
    nseg = 1 if seed % 3 else 3
    n_inputs = int(rng.integers(1, 4))
    kinds = ["full"] + [["full", "row", "col"][int(rng.integers(0, 3))] for _ in range(n_inputs - 1)]
    prog, n_out = _program(rng, n_inputs)
    reduce = ["none", "all", "rows", "cols"][int(rng.integers(0, 4))]
    mean = bool(rng.integers(0, 2)) and reduce != "none"
    if reduce == "none" and n_out == 0:
        prog.append(("STORE", "ACC", 0))
        n_out = 1

    host, views, devs = [], [], []
    for kind in kinds:
        shape = {"full": (nseg, rows, cols), "row": (nseg, 1, cols), "col": (nseg, rows, 1)}[kind]
        a = rng.uniform(-2, 2, shape).astype(np.float32)
        d = ttc.DeviceArray.from_numpy(a)
        devs.append(d)
        host.append(np.broadcast_to(a, (nseg, rows, cols)).astype(np.float32))
        if kind == "full":
            views.append(ttc.in_view(d.ptr, cols, 1, rows * cols))
        elif kind == "row":
            views.append(ttc.in_view(d.ptr, 0, 1, cols))
        else:
            views.append(ttc.in_view(d.ptr, 1, 0, rows))
    outs = [ttc.DeviceArray.empty((nseg, rows, cols)) for _ in range(n_out)]
    n_red = {"none": 0, "all": 1, "rows": rows, "cols": cols}[reduce]
    red = ttc.DeviceArray.empty((nseg, max(n_red, 1)))
    code = {"LOAD": ttc.OP_LOAD, "RELU": ttc.OP_RELU, "SIGMOID": ttc.OP_SIGMOID, "ADD": ttc.OP_ADD,
            "MUL": ttc.OP_MUL, "SAVE": ttc.OP_SAVE, "STORE": ttc.OP_STORE}
    srcs = {"ACC": ttc.SRC_ACC, "INPUT": ttc.SRC_INPUT, "SLOT": ttc.SRC_SLOT}
    instrs = [ttc.instr(code[op], srcs[src], idx) for op, src, idx in prog]
    mode = {"none": ttc.REDUCE_NONE, "all": ttc.REDUCE_ALL, "rows": ttc.REDUCE_ROWS,
            "cols": ttc.REDUCE_COLS}[reduce]
    desc = ttc.chain_desc(rows, cols, views, [ttc.out_view(o.ptr, cols, rows * cols) for o in outs], instrs,
                          reduce=mode, reduce_out=red.ptr if reduce != "none" else None, mean=mean, nseg=nseg,
                          reduce_seg_stride=max(n_red, 1))
    ttc.eltwise_chain(desc)

    acc, want_outs = _evaluate(prog, host)
    # sigmoid is exact against this host's formula unless its glibc is the
    # build without FMA (oracle.sigmoid_ulp_bound)
    has_sigmoid = any(op == "SIGMOID" for op, _, _ in prog) and oracle.sigmoid_ulp_bound() > 0
    for i in range(n_out):
        got, want = outs[i].numpy(), want_outs[i]
        both_nan = np.isnan(got) & np.isnan(want)
        assert np.array_equal(np.isnan(got), np.isnan(want)), prog
        if has_sigmoid:
            fin = np.isfinite(want)
            assert np.array_equal(got[~fin & ~both_nan], want[~fin & ~both_nan]), prog
            if fin.any():
                err = np.abs(got[fin].astype(np.float64) - want[fin]).max()
                assert err <= 1e-5 * max(1.0, float(np.abs(want[fin]).max())), (prog, err)
        else:
            same = both_nan | (got.view(np.int32) == want.view(np.int32))
            assert same.all(), prog
    if reduce != "none":
        a64 = acc.astype(np.float64)
        axis = {"all": (1, 2), "rows": 2, "cols": 1}[reduce]
        with np.errstate(invalid="ignore", over="ignore"):
            want = a64.sum(axis=axis)
            scale = np.abs(a64).sum(axis=axis) + 1e-30
        if mean:
            n = {"all": rows * cols, "rows": cols, "cols": rows}[reduce]
            want, scale = want / n, scale / n
        got = red.numpy().reshape(want.shape).astype(np.float64)
        fin = np.isfinite(want) & np.isfinite(scale) & (np.abs(want) < 3e38)
        assert (np.abs(got[fin] - want[fin]) <= 1e-5 * scale[fin]).all(), (prog, reduce)
        nan = np.isnan(want)
        assert np.isnan(got[nan]).all(), (prog, reduce)


def test_random_chains_on_the_staged_interpreter():
    """The programs above with the specialised kernels switched off
    (TTC_CHAIN_JIT=0, read once per process, so in a fresh one): the layouts
    of 1 Mi elements and more run on the TMA-staged interpreter."""
    env = dict(os.environ, TTC_CHAIN_JIT="0")
    r = subprocess.run([sys.executable, "-m", "pytest", __file__, "-q", "-x", "-p", "no:cacheprovider", "-k",
                        "test_random_chain_matches_oracle"], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
