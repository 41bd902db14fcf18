"""CPU oracle for the tt_lazy B200 backend -- TEST INFRASTRUCTURE ONLY.

Two libraries, both loaded through ctypes:

* ``liboracle.so`` (``oracle.c``): a plain-C restatement of the reference's
  ``namespace math`` backend (src/backend/cpu/*.cpp of ayerofieiev-tt/tt_lazy),
  same operation order, IEEE single ops, no FMA contraction.
* ``_ref/libttref.so`` (``build_ref.sh`` + ``ref_capi.cpp``): the reference's
  own sources compiled unmodified, used to pin the restatement and as the
  timed CPU baseline.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package; the product (``tt_lazy_b200``) never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libttref.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


class OracleError(RuntimeError):
    """Shape error raised by the oracle (mirrors the reference's runtime_error)."""


def build(force: bool = False) -> str:
    """Compile oracle.c into liboracle.so (gcc, -O2 -ffp-contract=off)."""
    src = os.path.join(HERE, "oracle.c")
    if (not force and os.path.exists(ORACLE_SO)
            and os.path.getmtime(ORACLE_SO) >= os.path.getmtime(src)
            and os.path.getmtime(ORACLE_SO) >= os.path.getmtime(os.path.join(HERE, "oracle.h"))):
        return ORACLE_SO
    tmp = ORACLE_SO + ".tmp"
    subprocess.check_call(["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
                           "-std=c11", src, "-o", tmp, "-lm"])
    os.replace(tmp, ORACLE_SO)
    return ORACLE_SO


def build_ref(force: bool = False) -> str | None:
    """Compile the reference sources into _ref/libttref.so when they are present."""
    # the reference checkout: $TT_REFERENCE_ROOT, default "reference" beside this repository
    ref_root = os.environ.get("TT_REFERENCE_ROOT",
                              os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
    deps = [os.path.join(HERE, "ref_capi.cpp"), os.path.join(HERE, "build_ref.sh")]
    if not os.path.isdir(os.path.join(ref_root, "src", "backend", "cpu")):
        return REF_SO if os.path.exists(REF_SO) else None
    if (not force and os.path.exists(REF_SO)
            and all(os.path.getmtime(REF_SO) >= os.path.getmtime(d) for d in deps)):
        return REF_SO
    subprocess.check_call(["sh", os.path.join(HERE, "build_ref.sh")])
    return REF_SO


_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(ORACLE_SO)
        L.orc_last_error.restype = C.c_char_p
        L.orc_relu.argtypes = [_f32p, _f32p, C.c_size_t]
        L.orc_sigmoid.argtypes = [_f32p, _f32p, C.c_size_t]
        L.orc_expf_ref.argtypes = [_f32p, _f32p, C.c_size_t]
        L.orc_expf_libm.argtypes = [_f32p, _f32p, C.c_size_t]
        for fn in (L.orc_add, L.orc_multiply):
            fn.argtypes = [_f32p, _u32p, C.c_int, _f32p, _u32p, C.c_int, _f32p]
        L.orc_matmul.argtypes = [_f32p, C.c_uint32, C.c_uint32, _f32p, C.c_uint32, C.c_uint32,
                                 C.c_int, C.c_int, _f32p]
        L.orc_fused_mlp.argtypes = [_f32p, _f32p, _f32p, C.c_uint32, C.c_uint32, C.c_uint32,
                                    C.c_int, _f32p]
        L.orc_reduce.argtypes = [_f32p, _u32p, C.c_int, _i32p, C.c_int, C.c_int, _f32p]
        L.orc_reduce_f64.argtypes = [_f32p, _u32p, C.c_int, _i32p, C.c_int, C.c_int, _f64p]
        L.orc_transpose.argtypes = [_f32p, _u32p, C.c_int, _f32p]
        L.orc_split_chunk.argtypes = [_f32p, _u32p, C.c_int, C.c_int64, C.c_int32, C.c_uint32, _f32p]
        _lib = L
    return _lib


def ref():
    """The reference compiled from its sources, or None when it was not built."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            return None
        L = C.CDLL(REF_SO)
        L.ref_last_error.restype = C.c_char_p
        L.ref_quiet()
        _ref = L
    return _ref


def _chk(rc, L, getter="orc_last_error"):
    if rc != 0:
        raise OracleError(getattr(L, getter)().decode())


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _shape(x):
    return np.asarray(x.shape, dtype=np.uint32)


# ---------------------------------------------------------------- restatement
def relu(x):
    x = _f32(x)
    out = np.empty_like(x)
    _chk(lib().orc_relu(x.reshape(-1), out.reshape(-1), x.size), lib())
    return out


def sigmoid(x):
    x = _f32(x)
    out = np.empty_like(x)
    _chk(lib().orc_sigmoid(x.reshape(-1), out.reshape(-1), x.size), lib())
    return out


def expf_ref(x):
    """glibc's expf restated as its x86-64 FMA build computes it (oracle.c)."""
    x = _f32(x)
    out = np.empty_like(x)
    _chk(lib().orc_expf_ref(x.reshape(-1), out.reshape(-1), x.size), lib())
    return out


def expf_libm(x):
    """This process's own expf (what the reference's std::exp(float) calls)."""
    x = _f32(x)
    out = np.empty_like(x)
    _chk(lib().orc_expf_libm(x.reshape(-1), out.reshape(-1), x.size), lib())
    return out


def expf_is_fma_build() -> bool:
    """True when this process's expf is glibc's FMA build. The device sigmoid
    equals the reference's on every float then; with glibc's other x86-64
    build one float of sigmoid differs by 1 ulp."""
    return bool(lib().orc_expf_is_fma_build())


def sigmoid_ulp_bound() -> int:
    """Largest ulp distance the tests allow between the device sigmoid and
    sigmoid() on this host: 0 where the host's expf is glibc's FMA build."""
    return 0 if expf_is_fma_build() else 1


def _binary(fn, a, b):
    a, b = _f32(a), _f32(b)
    shape = np.broadcast_shapes(a.shape, b.shape) if a.ndim and b.ndim else a.shape
    out = np.empty(shape, dtype=np.float32)
    _chk(fn(a.reshape(-1), _shape(a), a.ndim, b.reshape(-1), _shape(b), b.ndim, out.reshape(-1)), lib())
    return out


def add(a, b):
    return _binary(lib().orc_add, a, b)


def multiply(a, b):
    return _binary(lib().orc_multiply, a, b)


def matmul(a, b, transpose_a=False, transpose_b=False):
    a, b = _f32(a), _f32(b)
    m = a.shape[1] if transpose_a else a.shape[0]
    n = b.shape[0] if transpose_b else b.shape[1]
    out = np.empty((m, n), dtype=np.float32)
    _chk(lib().orc_matmul(a.reshape(-1), a.shape[0], a.shape[1], b.reshape(-1), b.shape[0], b.shape[1],
                          int(transpose_a), int(transpose_b), out.reshape(-1)), lib())
    return out


def fused_mlp(x, w, bias, has_relu=True):
    x, w, bias = _f32(x), _f32(w), _f32(bias)
    out = np.empty((x.shape[0], w.shape[1]), dtype=np.float32)
    _chk(lib().orc_fused_mlp(x.reshape(-1), w.reshape(-1), bias.reshape(-1), x.shape[0], x.shape[1],
                             w.shape[1], int(has_relu), out.reshape(-1)), lib())
    return out


def _reduced_shape(shape, dims, keepdim):
    rank = len(shape)
    red = set(range(rank)) if not dims else {d % rank for d in dims}
    out = [1 if i in red else s for i, s in enumerate(shape) if keepdim or i not in red]
    return tuple(out) if out else (1,)


def reduce(x, dims=(), keepdim=False, mean=False, f64=False):
    x = _f32(x)
    dims_a = np.asarray(list(dims), dtype=np.int32)
    shape = _reduced_shape(x.shape, list(dims), keepdim)
    if f64:
        out = np.empty(shape, dtype=np.float64)
        _chk(lib().orc_reduce_f64(x.reshape(-1), _shape(x), x.ndim, dims_a, len(dims_a), int(mean),
                                  out.reshape(-1)), lib())
    else:
        out = np.empty(shape, dtype=np.float32)
        _chk(lib().orc_reduce(x.reshape(-1), _shape(x), x.ndim, dims_a, len(dims_a), int(mean),
                              out.reshape(-1)), lib())
    return out


def reduce_sum(x, dims=(), keepdim=False):
    return reduce(x, dims, keepdim, mean=False)


def reduce_mean(x, dims=(), keepdim=False):
    return reduce(x, dims, keepdim, mean=True)


def transpose(x):
    x = _f32(x)
    shape = list(x.shape)
    shape[-2], shape[-1] = shape[-1], shape[-2]
    out = np.empty(shape, dtype=np.float32)
    _chk(lib().orc_transpose(x.reshape(-1), _shape(x), x.ndim, out.reshape(-1)), lib())
    return out


def split(x, split_size, dim=0):
    x = _f32(x)
    if split_size <= 0 or not 0 <= dim < x.ndim:
        scratch = np.empty(1, np.float32)
        _chk(lib().orc_split_chunk(x.reshape(-1), _shape(x), x.ndim, split_size, dim, 0, scratch), lib())
    size = x.shape[dim]
    n = (size + split_size - 1) // split_size
    outs = []
    for i in range(n):
        shape = list(x.shape)
        shape[dim] = min(split_size, size - i * split_size)
        out = np.empty(shape, dtype=np.float32)
        _chk(lib().orc_split_chunk(x.reshape(-1), _shape(x), x.ndim, split_size, dim, i, out.reshape(-1)), lib())
        outs.append(out)
    return outs


# ---------------------------------------------------------------- reference build
class Ref:
    """Thin numpy wrappers over oracle/_ref/libttref.so (the reference's code)."""

    def __init__(self):
        self.L = ref()
        if self.L is None:
            raise FileNotFoundError(REF_SO)

    def _c(self, rc):
        _chk(rc, self.L, "ref_last_error")

    def relu(self, x):
        x = _f32(x)
        out = np.empty_like(x)
        self._c(self.L.ref_math_relu(_p(x), _p(_shape(x)), x.ndim, _p(out)))
        return out

    def add(self, a, b):
        a, b = _f32(a), _f32(b)
        out = np.empty(np.broadcast_shapes(a.shape, b.shape), dtype=np.float32)
        self._c(self.L.ref_math_add(_p(a), _p(_shape(a)), a.ndim, _p(b), _p(_shape(b)), b.ndim, _p(out)))
        return out

    def multiply(self, a, b):
        a, b = _f32(a), _f32(b)
        out = np.empty(np.broadcast_shapes(a.shape, b.shape), dtype=np.float32)
        self._c(self.L.ref_math_multiply(_p(a), _p(_shape(a)), a.ndim, _p(b), _p(_shape(b)), b.ndim, _p(out)))
        return out

    def matmul(self, a, b, transpose_a=False, transpose_b=False):
        a, b = _f32(a), _f32(b)
        m = a.shape[1] if transpose_a else a.shape[0]
        n = b.shape[0] if transpose_b else b.shape[1]
        out = np.empty((m, n), dtype=np.float32)
        self._c(self.L.ref_math_matmul(_p(a), _p(_shape(a)), _p(b), _p(_shape(b)), int(transpose_a),
                                       int(transpose_b), _p(out)))
        return out

    def fused_mlp(self, x, w, b, has_relu=True):
        x, w, b = _f32(x), _f32(w), _f32(b)
        out = np.empty((x.shape[0], w.shape[1]), dtype=np.float32)
        self._c(self.L.ref_math_fused_mlp(_p(x), _p(_shape(x)), _p(w), _p(_shape(w)), _p(b), _p(_shape(b)),
                                          int(has_relu), _p(out)))
        return out

    def reduce_sum(self, x, dims=(), keepdim=False):
        """Raw reference result: (flat values, element count)."""
        x = _f32(x)
        d = np.asarray(list(dims), dtype=np.int32)
        out = np.zeros(x.size + 1, dtype=np.float32)
        n = C.c_size_t(0)
        self._c(self.L.ref_math_reduce_sum(_p(x), _p(_shape(x)), x.ndim, _p(d), len(d), int(keepdim), _p(out),
                                           C.c_size_t(out.size), C.byref(n)))
        return out[: n.value].copy()

    def transpose(self, x):
        x = _f32(x)
        shape = list(x.shape)
        shape[-2], shape[-1] = shape[-1], shape[-2]
        out = np.empty(shape, dtype=np.float32)
        self._c(self.L.ref_math_transpose(_p(x), _p(_shape(x)), x.ndim, _p(out)))
        return out

    def split_1d(self, x, split_size):
        x = _f32(x)
        out = np.empty(x.size, dtype=np.float32)
        self._c(self.L.ref_math_split_1d(_p(x), C.c_uint32(x.size), C.c_int64(split_size), _p(out)))
        return out

    def lazy_chain(self, x):
        x = _f32(x)
        out = np.empty_like(x)
        self._c(self.L.ref_lazy_chain(_p(x), _p(_shape(x)), x.ndim, _p(out)))
        return out

    def lazy_mlp2(self, x, w1, b1, w2, b2):
        arrs = [_f32(a) for a in (x, w1, b1, w2, b2)]
        out = np.empty((arrs[0].shape[0], arrs[3].shape[1]), dtype=np.float32)
        args = []
        for a in arrs:
            args += [_p(a), _p(_shape(a))]
        self._c(self.L.ref_lazy_mlp2(*args, _p(out)))
        return out

    def lazy_fused_mlp(self, x, w, b, has_relu=True):
        x, w, b = _f32(x), _f32(w), _f32(b)
        out = np.empty((x.shape[0], w.shape[1]), dtype=np.float32)
        self._c(self.L.ref_lazy_fused_mlp(_p(x), _p(_shape(x)), _p(w), _p(_shape(w)), _p(b), _p(_shape(b)),
                                          int(has_relu), _p(out)))
        return out


def _p(a):
    return a.ctypes.data_as(C.c_void_p)
