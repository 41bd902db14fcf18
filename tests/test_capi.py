"""The C-ABI library loads and exports every entry point include/tt_cuda.h
declares; calls made before ttc_init fail with a status, not a crash."""
import ctypes as C
import os
import re

from tt_lazy_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "tt_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ttc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = capi.lib()
    decl = declared_symbols()
    assert decl, "no declarations parsed"
    missing = [s for s in decl if not hasattr(L, s)]
    assert not missing, missing
    assert sorted(capi.EXPORTS) == decl


def test_calls_before_init_return_status():
    L = capi.lib()
    p = C.c_void_p()
    assert L.ttc_malloc(16, C.byref(p)) == capi.ERR_NOT_INIT
    assert b"ttc_init" in L.ttc_last_error()
    d = capi.ChainDesc()
    assert L.ttc_eltwise_chain(C.byref(d)) == capi.ERR_NOT_INIT
    assert L.ttc_version() >= 1


def test_injected_comm_faults_return_an_error_status(monkeypatch):
    """A failing communicator call (faked on the host, before NCCL or the GPU
    is touched) comes back as TTC_ERR_NCCL with a message, not a crash."""
    L = capi.lib()
    uid = bytes(128)
    monkeypatch.setenv("TTC_COMM_FAULT", "init")
    assert L.ttc_comm_init(2, 0, uid, 1000) == 6
    assert b"injected" in L.ttc_last_error()
    monkeypatch.setenv("TTC_COMM_FAULT", "allreduce")
    assert L.ttc_allreduce_sum(None, 0, 1000) == 6
    assert b"injected" in L.ttc_last_error()
    monkeypatch.delenv("TTC_COMM_FAULT")
    assert L.ttc_allreduce_sum(None, 0, 1000) == capi.ERR_NOT_INIT  # no communicator


def test_chain_jit_source_needs_no_device():
    I = capi.instr
    d = capi.chain_desc(64, 64, [capi.in_view(0x1000, 64)], [capi.out_view(0x2000, 64)],
                        [I(capi.OP_LOAD, idx=0), I(capi.OP_SIGMOID), I(capi.OP_STORE, idx=0)])
    src = capi.chain_jit_source(d)
    assert "ttj_sigmoid_all" in src and "ttj_flat<W, G, true, false, Body>" in src
    bad = capi.chain_desc(64, 64, [], [], [I(capi.OP_LOAD, idx=3)])
    n = C.c_size_t()
    assert capi.lib().ttc_chain_jit_source(C.byref(bad), None, 0, C.byref(n)) == 1
