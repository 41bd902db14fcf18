"""Failure detection inside the TMA-fed kernels, without faulting the GPU.

Every mbarrier wait of the tcgen05 GEMM kernels (single-CTA and CTA-pair)
and of the TMA-staged chain kernel is bounded. The test switch
TTC_TEST_STALL=gemm|chain (read at every launch) makes the kernel's TMA
producer issue no loads at all -- nothing is ever in flight -- and shortens
the limit to ~1 ms: the consumers' waits on the never-filled stages run out,
the kernel records the expiry in the host-mapped status word, frees its
tensor memory and returns, and the next synchronisation reports
TTC_ERR_TIMEOUT. The same context then runs the kernel normally and matches
the oracle."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _normwise(got, want):
    w = want.astype(np.float64)
    return np.linalg.norm(got.astype(np.float64) - w) / np.linalg.norm(w)


@pytest.mark.parametrize("pair", ["0", "1"])
def test_gemm_wait_expiry_is_reported_and_the_context_stays_usable(ttc, monkeypatch, pair):
    monkeypatch.setenv("TTC_GEMM_PAIR", pair)  # 1: the cta_group::2 kernel, 0: the single-CTA kernel
    rng = np.random.default_rng(17)
    M, N, K = 1024, 1024, 512
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = (rng.standard_normal((K, N)) / np.sqrt(K)).astype(np.float32)
    A, B = ttc.DeviceArray.from_numpy(a), ttc.DeviceArray.from_numpy(b)
    Cm = ttc.DeviceArray.empty((M, N))
    ttc.synchronize()
    monkeypatch.setenv("TTC_TEST_STALL", "gemm")
    ttc.gemm(M, N, K, A.ptr, K, B.ptr, N, Cm.ptr, N, path=ttc.GEMM_TF32)
    with pytest.raises(ttc.TTCError) as e:
        ttc.synchronize()
    assert e.value.code == ttc.ERR_TIMEOUT, str(e.value)
    assert "bounded wait expired" in str(e.value)
    monkeypatch.delenv("TTC_TEST_STALL")
    ttc.synchronize()  # the status word was cleared: nothing pending
    ttc.gemm(M, N, K, A.ptr, K, B.ptr, N, Cm.ptr, N, path=ttc.GEMM_TF32)
    ttc.synchronize()
    assert _normwise(Cm.numpy(), oracle.matmul(a, b)) <= 2e-3


_CHAIN = r"""
import ctypes as C, sys
import numpy as np
sys.path.insert(0, %r)
import oracle
from tt_lazy_b200 import capi as ttc
import os
ttc.init(0)
rows, cols = 2048, 1024   # 2 Mi elements: the staged kernel takes it with the specialised kernels off
x = np.random.default_rng(23).uniform(-2, 2, (rows, cols)).astype(np.float32)
X = ttc.DeviceArray.from_numpy(x)
Y = ttc.DeviceArray.empty((rows, cols))
prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_RELU), ttc.instr(ttc.OP_ADD, ttc.SRC_ACC),
        ttc.instr(ttc.OP_STORE, idx=0)]
d = ttc.chain_desc(rows, cols, [ttc.in_view(X.ptr, cols)], [ttc.out_view(Y.ptr, cols)], prog)
os.environ["TTC_TEST_STALL"] = "chain"
ttc.eltwise_chain(d)
try:
    ttc.synchronize()
    print("no timeout")
    sys.exit(1)
except ttc.TTCError as e:
    assert e.code == ttc.ERR_TIMEOUT, e
del os.environ["TTC_TEST_STALL"]
ttc.eltwise_chain(d)
ttc.synchronize()
r = oracle.relu(x)
ok = np.array_equal(Y.numpy(), oracle.add(r, r))
print("recovered_bit_exact=%%d" %% ok)
"""


def test_staged_chain_wait_expiry_is_reported_and_the_context_stays_usable():
    """The TMA-staged chain kernel runs only with the program-specialised
    kernels off (TTC_CHAIN_JIT=0, read once per process): a fresh process."""
    env = dict(os.environ, TTC_CHAIN_JIT="0")
    env.pop("TTC_TEST_STALL", None)
    r = subprocess.run([sys.executable, "-c", _CHAIN % ROOT], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "recovered_bit_exact=1" in r.stdout, r.stdout
