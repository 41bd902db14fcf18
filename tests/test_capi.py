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
