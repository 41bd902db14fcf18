"""ttc_eltwise_chain_noalloc: the element-wise chain entry point for callers
that cannot allocate device memory while they run -- a serving loop that
reserves all its memory at start-up (an allocation mid-request can stall or
fail), or a host framework whose own pool owns every device allocation. Its
reduction scratch is a fixed 1 MiB device array inside the library instead
of library-allocated memory.

Checked through the C-ABI against ttc_eltwise_chain on the same inputs, on
two calls in a row (the shared scratch keeps the previous call's contents),
within the reduction tolerance of the other parity tests (1e-5 relative).
This file runs last so a failure here stops a `-x` run only after every other
test has run; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _desc(ttc, X, rows, cols, out, mode, mean=False, nseg=1, seg_stride=0, out_seg=0):
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_SIGMOID), ttc.instr(ttc.OP_ADD, ttc.SRC_ACC)]
    return ttc.chain_desc(rows, cols, [ttc.in_view(X.ptr, cols, 1, seg_stride)], [], prog, reduce=mode,
                          reduce_out=out.ptr, mean=mean, nseg=nseg, reduce_seg_stride=out_seg)


@pytest.mark.parametrize("rows,cols,mode,nseg", [
    (2048, 3000, "all", 1),     # full sum: one partial per block
    (65536, 128, "cols", 1),    # column sums over many rows: split into row bands
    (4096, 4096, "cols", 1),
    (512, 1024, "cols", 4),     # segments
    (300, 777, "rows", 1),      # row sums: no partials
])
def test_noalloc_matches_allocating_entry_point(ttc, rows, cols, mode, nseg):
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
    before = ttc.stats()
    for _ in range(2):
        out = ttc.DeviceArray.empty((nseg, n_out))
        d = _desc(ttc, X, rows, cols, out, red, nseg=nseg, seg_stride=rows * cols, out_seg=n_out)
        ttc.check(L.ttc_eltwise_chain_noalloc(C.byref(d)))
        got = out.numpy()
        assert np.allclose(got, want, rtol=RTOL, atol=1e-6), np.max(np.abs(got - want) / np.abs(want))
    after = ttc.stats()
    # nothing allocated through the library while the entry point ran (the
    # two output buffers above are the test's own ttc_malloc calls)
    assert after.workspace_bytes == before.workspace_bytes


def test_noalloc_rejects_bad_descriptor(ttc):
    L = ttc.lib()
    X = ttc.DeviceArray.empty((4, 4))
    d = ttc.chain_desc(4, 4, [ttc.in_view(X.ptr, 4)], [], [ttc.instr(ttc.OP_RELU)])
    assert L.ttc_eltwise_chain_noalloc(C.byref(d)) == ttc.ERR_INVALID
    assert L.ttc_last_error()
