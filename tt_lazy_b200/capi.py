"""ctypes binding of the tt_cuda_lib C-ABI (``include/tt_cuda.h``).

This is the same boundary a C or C++ caller uses: device pointers, sizes and
strides, an int status. Every non-zero status raises :class:`TTCError` with
the library's ``ttc_last_error()`` text. The library is loaded from the
in-tree build (``tt_lazy_b200/lib/libtt_cuda.so``); a missing library is an
ImportError, never a silent fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libtt_cuda.so")

MAX_INPUTS, MAX_OUTPUTS, MAX_INSTR, SLOTS = 6, 4, 32, 4

# ttc_status
OK, ERR_INVALID, ERR_CUDA, ERR_OOM, ERR_UNSUPPORTED, ERR_NOT_INIT, ERR_NCCL, ERR_TIMEOUT = range(8)
# ttc_opcode
OP_LOAD, OP_RELU, OP_SIGMOID, OP_ADD, OP_MUL, OP_SAVE, OP_STORE = range(1, 8)
# ttc_src_kind
SRC_ACC, SRC_INPUT, SRC_SLOT = range(3)
# ttc_reduce_mode
REDUCE_NONE, REDUCE_ALL, REDUCE_ROWS, REDUCE_COLS = range(4)
# ttc_gemm_path
GEMM_AUTO, GEMM_FFMA, GEMM_TF32, GEMM_TF32X3 = range(4)


class Instr(C.Structure):
    _fields_ = [("op", C.c_uint8), ("src", C.c_uint8), ("idx", C.c_uint8), ("pad", C.c_uint8)]


class InView(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("row_stride", C.c_int64), ("col_stride", C.c_int64),
                ("seg_stride", C.c_int64)]


class OutView(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("row_stride", C.c_int64), ("seg_stride", C.c_int64)]


class ChainDesc(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("nseg", C.c_int32),
                ("n_inputs", C.c_int32), ("n_outputs", C.c_int32), ("n_instr", C.c_int32),
                ("inputs", InView * MAX_INPUTS), ("outputs", OutView * MAX_OUTPUTS),
                ("program", Instr * MAX_INSTR),
                ("reduce", C.c_int32), ("reduce_mean", C.c_int32),
                ("reduce_out", C.c_void_p), ("reduce_seg_stride", C.c_int64)]


class GemmDesc(C.Structure):
    _fields_ = [("M", C.c_int32), ("N", C.c_int32), ("K", C.c_int32),
                ("a", C.c_void_p), ("lda", C.c_int64), ("trans_a", C.c_int32),
                ("b", C.c_void_p), ("ldb", C.c_int64), ("trans_b", C.c_int32),
                ("c", C.c_void_p), ("ldc", C.c_int64),
                ("path", C.c_int32),
                ("epilogue", ChainDesc)]


class MemoryStats(C.Structure):
    _fields_ = [("bytes_in_use", C.c_size_t), ("peak_bytes", C.c_size_t), ("workspace_bytes", C.c_size_t),
                ("kernels_launched", C.c_uint64)]


# Every symbol include/tt_cuda.h declares (checked by tests/test_capi.py).
EXPORTS = ["ttc_last_error", "ttc_init", "ttc_shutdown", "ttc_device_count", "ttc_version", "ttc_get_stream",
           "ttc_set_stream", "ttc_synchronize", "ttc_malloc", "ttc_free", "ttc_memcpy_h2d", "ttc_memcpy_d2h", "ttc_h2d_prefetch", "ttc_wait_ticket", "ttc_capture_begin", "ttc_capture_end", "ttc_graph_launch", "ttc_graph_destroy", "ttc_range_push", "ttc_range_pop", "ttc_timer_mark", "ttc_timer_elapsed",
           "ttc_memcpy_d2d", "ttc_memset_zero", "ttc_host_alloc", "ttc_host_free", "ttc_get_memory_stats",
           "ttc_eltwise_chain", "ttc_eltwise_chain_noalloc", "ttc_chain_jit_source", "ttc_reduce", "ttc_transpose", "ttc_copy2d", "ttc_gemm", "ttc_gemm_select_path",
           "ttc_comm_unique_id", "ttc_comm_init", "ttc_allreduce_sum", "ttc_comm_destroy"]


class TTCError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


_lib = None


def lib():
    """Load libtt_cuda.so (raises ImportError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"tt_cuda library not built: {LIB_PATH} (run python tt_lazy_b200/build.py)")
        L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        L.ttc_last_error.restype = C.c_char_p
        L.ttc_get_stream.restype = C.c_void_p
        L.ttc_malloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)]
        L.ttc_free.argtypes = [C.c_void_p]
        for fn in (L.ttc_memcpy_h2d, L.ttc_memcpy_d2h, L.ttc_memcpy_d2d):
            fn.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t]
        L.ttc_memset_zero.argtypes = [C.c_void_p, C.c_size_t]
        L.ttc_h2d_prefetch.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]
        L.ttc_wait_ticket.argtypes = [C.c_int]
        L.ttc_capture_end.argtypes = [C.POINTER(C.c_void_p)]
        L.ttc_graph_launch.argtypes = [C.c_void_p]
        L.ttc_graph_destroy.argtypes = [C.c_void_p]
        L.ttc_range_push.argtypes = [C.c_char_p]
        L.ttc_timer_mark.argtypes = [C.POINTER(C.c_int)]
        L.ttc_timer_elapsed.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_float)]
        L.ttc_host_alloc.argtypes = [C.c_size_t, C.POINTER(C.c_void_p)]
        L.ttc_host_free.argtypes = [C.c_void_p]
        L.ttc_set_stream.argtypes = [C.c_void_p]
        L.ttc_eltwise_chain.argtypes = [C.POINTER(ChainDesc)]
        L.ttc_eltwise_chain_noalloc.argtypes = [C.POINTER(ChainDesc)]
        L.ttc_chain_jit_source.argtypes = [C.POINTER(ChainDesc), C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]
        L.ttc_gemm.argtypes = [C.POINTER(GemmDesc)]
        L.ttc_gemm_select_path.argtypes = [C.POINTER(GemmDesc)]
        L.ttc_reduce.argtypes = [C.c_void_p, C.POINTER(C.c_uint32), C.c_int, C.POINTER(C.c_int32), C.c_int,
                                 C.c_int, C.c_void_p]
        L.ttc_transpose.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64]
        L.ttc_copy2d.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_int64, C.c_int64]
        L.ttc_get_memory_stats.argtypes = [C.POINTER(MemoryStats)]
        L.ttc_allreduce_sum.argtypes = [C.c_void_p, C.c_size_t, C.c_int]
        L.ttc_comm_init.argtypes = [C.c_int, C.c_int, C.c_char_p, C.c_int]
        L.ttc_comm_unique_id.argtypes = [C.c_char_p]
        _lib = L
    return _lib


def check(rc):
    if rc != OK:
        raise TTCError(rc, lib().ttc_last_error().decode())
    return rc


def init(device=0):
    check(lib().ttc_init(device))


def synchronize():
    check(lib().ttc_synchronize())


def stats() -> MemoryStats:
    s = MemoryStats()
    check(lib().ttc_get_memory_stats(C.byref(s)))
    return s


def kernels_launched() -> int:
    return int(stats().kernels_launched)


class DeviceArray:
    """A float32 buffer in device memory, owned through ttc_malloc/ttc_free."""

    def __init__(self, shape, ptr=None, owner=True):
        self.shape = tuple(int(s) for s in shape)
        self.size = int(np.prod(self.shape)) if self.shape else 1
        self.nbytes = self.size * 4
        if ptr is None:
            p = C.c_void_p()
            check(lib().ttc_malloc(self.nbytes, C.byref(p)))
            ptr = p.value
        self.ptr = ptr
        self._owner = owner

    @classmethod
    def from_numpy(cls, a):
        a = np.ascontiguousarray(a, dtype=np.float32)
        d = cls(a.shape)
        check(lib().ttc_memcpy_h2d(d.ptr, a.ctypes.data, d.nbytes))
        return d

    @classmethod
    def empty(cls, shape):
        return cls(shape)

    @classmethod
    def zeros(cls, shape):
        d = cls(shape)
        check(lib().ttc_memset_zero(d.ptr, d.nbytes))
        return d

    def numpy(self):
        out = np.empty(self.shape, dtype=np.float32)
        check(lib().ttc_memcpy_d2h(out.ctypes.data, self.ptr, self.nbytes))
        return out

    def at(self, elem_offset):
        """Pointer to element `elem_offset` (a view; no ownership)."""
        return (self.ptr or 0) + 4 * int(elem_offset)

    def free(self):
        if self._owner and self.ptr:
            lib().ttc_free(self.ptr)
        self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ------------------------------------------------------------ descriptor helpers
def in_view(ptr, row_stride, col_stride=1, seg_stride=0):
    return InView(ptr, row_stride, col_stride, seg_stride)


def out_view(ptr, row_stride, seg_stride=0):
    return OutView(ptr, row_stride, seg_stride)


def instr(op, src=SRC_ACC, idx=0):
    return Instr(op, src, idx, 0)


def chain_desc(rows, cols, inputs, outputs, program, reduce=REDUCE_NONE, reduce_out=None, mean=False, nseg=1,
               reduce_seg_stride=0):
    d = ChainDesc()
    d.rows, d.cols, d.nseg = rows, cols, nseg
    d.n_inputs, d.n_outputs, d.n_instr = len(inputs), len(outputs), len(program)
    for i, v in enumerate(inputs):
        d.inputs[i] = v
    for i, v in enumerate(outputs):
        d.outputs[i] = v
    for i, v in enumerate(program):
        d.program[i] = v
    d.reduce = reduce
    d.reduce_mean = int(mean)
    d.reduce_out = reduce_out
    d.reduce_seg_stride = reduce_seg_stride
    return d


def eltwise_chain(desc):
    check(lib().ttc_eltwise_chain(C.byref(desc)))


def chain_jit_source(desc):
    """CUDA source of the specialised kernel for `desc` (no device needed)."""
    n = C.c_size_t(0)
    check(lib().ttc_chain_jit_source(C.byref(desc), None, 0, C.byref(n)))
    buf = C.create_string_buffer(n.value + 1)
    check(lib().ttc_chain_jit_source(C.byref(desc), buf, n.value + 1, C.byref(n)))
    return buf.value.decode()


def gemm(M, N, K, a, lda, b, ldb, c=None, ldc=0, trans_a=False, trans_b=False, path=GEMM_AUTO, epilogue=None):
    g = GemmDesc()
    g.M, g.N, g.K = M, N, K
    g.a, g.lda, g.trans_a = a, lda, int(trans_a)
    g.b, g.ldb, g.trans_b = b, ldb, int(trans_b)
    g.c, g.ldc = c, ldc
    g.path = path
    if epilogue is not None:
        g.epilogue = epilogue
    check(lib().ttc_gemm(C.byref(g)))
    return g


def gemm_select_path(g) -> int:
    return lib().ttc_gemm_select_path(C.byref(g))


def reduce(in_ptr, shape, dims, mean, out_ptr):
    sh = (C.c_uint32 * len(shape))(*shape)
    dd = (C.c_int32 * max(1, len(dims)))(*dims)
    check(lib().ttc_reduce(in_ptr, sh, len(shape), dd, len(dims), int(mean), out_ptr))


def transpose(in_ptr, out_ptr, batch, rows, cols):
    check(lib().ttc_transpose(in_ptr, out_ptr, batch, rows, cols))


def copy2d(in_ptr, in_ld, out_ptr, out_ld, rows, cols):
    check(lib().ttc_copy2d(in_ptr, in_ld, out_ptr, out_ld, rows, cols))
