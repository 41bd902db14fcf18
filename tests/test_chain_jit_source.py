"""The program-specialised chain kernels compile for sm_100a: the source that
ttc_chain_jit_source returns (exactly what the library hands to NVRTC at
first use) is compiled here with NVRTC and the library's options, for the
chain shapes the front end produces. NVRTC needs no GPU."""
import ctypes as C
import os
import re

import pytest

from tt_lazy_b200 import capi as ttc

I = ttc.instr
P = 0x10000  # any 16-byte aligned address: the source does not depend on it


def _nvrtc():
    for name in ("libnvrtc.so.12", "/usr/local/cuda/lib64/libnvrtc.so.12"):
        try:
            return C.CDLL(name)
        except OSError:
            pass
    pytest.skip("NVRTC not available")


def compile_source(src):
    L = _nvrtc()
    prog = C.c_void_p()
    assert L.nvrtcCreateProgram(C.byref(prog), src.encode(), b"ttc_chain_jit.cu", 0, None, None) == 0
    opts = [b"--gpu-architecture=sm_100a", b"-fmad=false", b"--std=c++17", b"-lineinfo", b"--ptxas-options=-v"]
    arr = (C.c_char_p * len(opts))(*opts)
    rc = L.nvrtcCompileProgram(prog, len(opts), arr)
    n = C.c_size_t()
    L.nvrtcGetProgramLogSize(prog, C.byref(n))
    log = C.create_string_buffer(n.value + 1)
    L.nvrtcGetProgramLog(prog, log)
    size = C.c_size_t()
    L.nvrtcGetCUBINSize(prog, C.byref(size))
    L.nvrtcDestroyProgram(C.byref(prog))
    return rc, log.value.decode(errors="replace"), size.value


def cases():
    N = 4096
    full = ttc.in_view(P, N)
    yield "copy", ttc.chain_desc(N, N, [full], [ttc.out_view(P, N)], [I(ttc.OP_LOAD, idx=0), I(ttc.OP_STORE, idx=0)])
    # README chain: relu -> add -> multiply, stored and summed
    yield "readme", ttc.chain_desc(N, N, [full], [ttc.out_view(P, N)],
                                   [I(ttc.OP_LOAD, idx=0), I(ttc.OP_RELU), I(ttc.OP_ADD, ttc.SRC_ACC),
                                    I(ttc.OP_MUL, ttc.SRC_ACC), I(ttc.OP_STORE, idx=0)],
                                   reduce=ttc.REDUCE_ALL, reduce_out=P)
    # bandwidth graph: sigmoid(C) * relu(C + C) over 8 segments, column sums
    yield "segments", ttc.chain_desc(N // 8, N, [ttc.in_view(P, N, 1, N * N // 8)], [],
                                     [I(ttc.OP_LOAD, idx=0), I(ttc.OP_ADD, ttc.SRC_ACC), I(ttc.OP_RELU),
                                      I(ttc.OP_SAVE, idx=0), I(ttc.OP_LOAD, idx=0), I(ttc.OP_SIGMOID),
                                      I(ttc.OP_MUL, ttc.SRC_SLOT, 0)],
                                     reduce=ttc.REDUCE_COLS, reduce_out=P, nseg=8, reduce_seg_stride=N)
    # bias row broadcast + relu, two inputs, row sums
    yield "bias_rows", ttc.chain_desc(N, N, [full, ttc.in_view(P, 0)], [],
                                      [I(ttc.OP_LOAD, idx=0), I(ttc.OP_ADD, ttc.SRC_INPUT, 1), I(ttc.OP_RELU)],
                                      reduce=ttc.REDUCE_ROWS, reduce_out=P)
    # three inputs including a column broadcast, two stored outputs
    yield "three_inputs", ttc.chain_desc(N, N, [full, full, ttc.in_view(P, 1, 0)],
                                         [ttc.out_view(P, N), ttc.out_view(P, N)],
                                         [I(ttc.OP_LOAD, idx=0), I(ttc.OP_MUL, ttc.SRC_INPUT, 1), I(ttc.OP_STORE, idx=0),
                                          I(ttc.OP_SIGMOID), I(ttc.OP_ADD, ttc.SRC_INPUT, 2), I(ttc.OP_STORE, idx=1)])


@pytest.mark.parametrize("name,desc", list(cases()), ids=[c[0] for c in cases()])
def test_specialised_source_compiles_without_spills(name, desc):
    src = ttc.chain_jit_source(desc)
    assert "ttj_kernel" in src and "struct Body" in src
    rc, log, size = compile_source(src)
    assert rc == 0, log
    assert size > 0
    spills = [int(x) for x in re.findall(r"(\d+) bytes spill stores", log)]
    assert spills and max(spills) == 0, log
    regs = [int(x) for x in re.findall(r"Used (\d+) registers", log)]
    assert regs and max(regs) <= 128, log
