"""ttc_eltwise_chain_noalloc: the element-wise chain entry point for callers
that cannot allocate device memory while they run -- a serving loop that
reserves all its memory at start-up (an allocation mid-request can stall or
fail), or a host framework whose own pool owns every device allocation. Its
reduction scratch is a fixed 1 MiB device array inside the library instead
of library-allocated memory.

Checked through the C-ABI against ttc_eltwise_chain on the same inputs, on
two calls in a row (the shared scratch keeps the previous call's contents),
within the reduction tolerance of the other parity tests (1e-5 relative), and
against the oracle (the fp64 sum of the oracle's element values). A wide
column sum whose row bands would not all fit in the array runs with fewer
bands; a fresh process whose first chain call is this entry point allocates
no library scratch. This file runs last so a failure here stops a `-x` run
only after every other test has run; it also passes alone in a fresh process.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

RTOL = 1e-5
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _desc(ttc, X, rows, cols, out, mode, mean=False, nseg=1, seg_stride=0, out_seg=0):
    # acc = sigmoid(x) + sigmoid(x), reduced
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_SIGMOID), ttc.instr(ttc.OP_ADD, ttc.SRC_ACC)]
    return ttc.chain_desc(rows, cols, [ttc.in_view(X.ptr, cols, 1, seg_stride)], [], prog, reduce=mode,
                          reduce_out=out.ptr, mean=mean, nseg=nseg, reduce_seg_stride=out_seg)


def _oracle_sums(x, nseg, rows, cols, mode):
    s = oracle.sigmoid(x)
    v = oracle.add(s, s).astype(np.float64).reshape(nseg, rows, cols)
    a = np.abs(v)
    axis = {"all": (1, 2), "cols": 1, "rows": 2}[mode]
    return v.sum(axis=axis).reshape(nseg, -1), a.sum(axis=axis).reshape(nseg, -1)


@pytest.mark.parametrize("rows,cols,mode,nseg", [
    (2048, 3000, "all", 1),     # full sum: one partial per block
    (65536, 128, "cols", 1),    # column sums over many rows: split into row bands
    (4096, 4096, "cols", 1),
    (512, 1024, "cols", 4),     # segments
    (300, 777, "rows", 1),      # row sums: no partials
    (512, 140000, "cols", 1),   # wide: row bands limited by the array (one band)
])
def test_noalloc_matches_allocating_entry_point_and_oracle(ttc, rows, cols, mode, nseg):
    L = ttc.lib()
    rng = np.random.default_rng(7)
    x = rng.uniform(-2, 2, (nseg * rows, cols)).astype(np.float32)
    X = ttc.DeviceArray.from_numpy(x)
    red = {"all": ttc.REDUCE_ALL, "cols": ttc.REDUCE_COLS, "rows": ttc.REDUCE_ROWS}[mode]
    n_out = {"all": 1, "cols": cols, "rows": rows}[mode]
    ref = ttc.DeviceArray.empty((nseg, n_out))
    d_ref = _desc(ttc, X, rows, cols, ref, red, nseg=nseg, seg_stride=rows * cols, out_seg=n_out)
    ttc.check(L.ttc_eltwise_chain(C.byref(d_ref)))
    want = ref.numpy()
    exact, scale = _oracle_sums(x, nseg, rows, cols, mode)
    before = ttc.stats()
    for _ in range(2):
        out = ttc.DeviceArray.empty((nseg, n_out))
        d = _desc(ttc, X, rows, cols, out, red, nseg=nseg, seg_stride=rows * cols, out_seg=n_out)
        ttc.check(L.ttc_eltwise_chain_noalloc(C.byref(d)))
        got = out.numpy()
        assert np.allclose(got, want, rtol=RTOL, atol=1e-6), np.max(np.abs(got - want) / np.abs(want))
        assert np.all(np.abs(got - exact) <= RTOL * scale), np.max(np.abs(got - exact) / scale)
    after = ttc.stats()
    assert after.workspace_bytes == before.workspace_bytes


_FRESH = r"""
import ctypes as C, numpy as np, sys
sys.path.insert(0, %r)
from tt_lazy_b200 import capi as ttc
ttc.init(0)
L = ttc.lib()
rows, cols = 8192, 512
x = np.random.default_rng(3).uniform(-2, 2, (rows, cols)).astype(np.float32)
X = ttc.DeviceArray.from_numpy(x)
outs = []
for mode, n in ((ttc.REDUCE_COLS, cols), (ttc.REDUCE_ALL, 1)):
    out = ttc.DeviceArray.empty((n,))
    d = ttc.chain_desc(rows, cols, [ttc.in_view(X.ptr, cols)], [], [ttc.instr(ttc.OP_LOAD, idx=0),
                       ttc.instr(ttc.OP_SIGMOID)], reduce=mode, reduce_out=out.ptr)
    ttc.check(L.ttc_eltwise_chain_noalloc(C.byref(d)))
    outs.append(out.numpy())
ws = ttc.stats().workspace_bytes
print("workspace_bytes=%%d cols0=%%.9g total=%%.9g" %% (ws, outs[0][0], outs[1][0]))
"""


def test_noalloc_first_in_a_fresh_process_allocates_no_scratch():
    """A process whose first chain calls are this entry point (a column sum
    that splits into row bands and a full sum, both with partials) never
    grows the library's scratch workspace."""
    r = subprocess.run([sys.executable, "-c", _FRESH % ROOT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("workspace_bytes=")][-1]
    assert line.split()[0] == "workspace_bytes=0", line
    x = np.random.default_rng(3).uniform(-2, 2, (8192, 512)).astype(np.float32)
    s = oracle.sigmoid(x).astype(np.float64)
    col0, total = (float(v.split("=")[1]) for v in line.split()[1:])
    assert abs(col0 - s[:, 0].sum()) <= RTOL * s[:, 0].sum()
    assert abs(total - s.sum()) <= RTOL * s.sum()


def test_noalloc_rejects_bad_descriptor(ttc):
    L = ttc.lib()
    X = ttc.DeviceArray.empty((4, 4))
    d = ttc.chain_desc(4, 4, [ttc.in_view(X.ptr, 4)], [], [ttc.instr(ttc.OP_RELU)])
    assert L.ttc_eltwise_chain_noalloc(C.byref(d)) == ttc.ERR_INVALID
    assert L.ttc_last_error()
