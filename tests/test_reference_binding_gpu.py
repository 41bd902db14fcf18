"""The reference-side binding, compiled and run: the reference's own front
end and tape (src/core, src/frontend, src/tape of ayerofieiev-tt/tt_lazy,
unmodified) with tt_lazy_b200/binding/OperationHandlers.cpp as their
operation handlers, linked to libtt_cuda.so instead of the CPU library
(tests/native/build_reference_binding.sh builds it). The reference's
Tensor::to_vector() evaluates through its TapeEvaluationManager and
TapeExecutor into the binding's handlers and the CUDA backend; results are
checked against the oracle with the usual bounds (element-wise bit-exact,
sums 1e-5 relative to the fp64 sum, matmul norm-wise 1e-5 on the FFMA and
TF32X3 paths, 2e-3 on TF32)."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "native", "_build", "libttref_cuda.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")


@pytest.fixture(scope="module")
def rb():
    if not os.path.exists(SO):
        pytest.skip("reference binding not built (needs the reference sources at build time)")
    L = C.CDLL(SO)  # finds tt_lazy_b200/lib/libtt_cuda.so through its run path
    L.rb_last_error.restype = C.c_char_p
    L.rb_readme_chain.argtypes = [_f32p, C.c_uint32, C.c_uint32, _f32p, _f32p]
    L.rb_mlp2.argtypes = [_f32p, C.c_uint32, C.c_uint32, _f32p, C.c_uint32, _f32p, _f32p, C.c_uint32, _f32p,
                          _f32p]
    L.rb_row_sums.argtypes = [_f32p, C.c_uint32, C.c_uint32, _f32p]
    L.rb_bad_broadcast.argtypes = [_f32p, C.c_uint32, C.c_uint32, _f32p]
    return L


def _ok(L, rc):
    assert rc == 0, L.rb_last_error().decode()


def test_readme_chain_through_the_reference_front_end(rb):
    x = np.random.default_rng(0).uniform(-1, 1, (1000, 1000)).astype(np.float32)
    w = np.empty_like(x)
    s = np.empty(1, np.float32)
    _ok(rb, rb.rb_readme_chain(x, 1000, 1000, w, s))
    r = oracle.relu(x)
    z = oracle.add(r, r)
    want = oracle.multiply(z, z)
    assert np.array_equal(w.view(np.int32), want.view(np.int32))
    exact = want.astype(np.float64).sum()
    assert abs(s[0] - exact) <= 1e-5 * exact


@pytest.mark.parametrize("path,tol", [("ffma", 1e-5), ("tf32x3", 1e-5), ("tf32", 2e-3)])
def test_two_layer_mlp_through_the_reference_front_end(rb, monkeypatch, path, tol):
    monkeypatch.setenv("TT_LAZY_GEMM", path)  # the binding reads it at every matmul
    rng = np.random.default_rng(1)
    X = rng.standard_normal((256, 512)).astype(np.float32)
    W1 = (rng.standard_normal((512, 1024)) / np.sqrt(512)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, (1, 1024)).astype(np.float32)
    W2 = (rng.standard_normal((1024, 512)) / np.sqrt(1024)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, (1, 512)).astype(np.float32)
    y = np.empty((256, 512), np.float32)
    _ok(rb, rb.rb_mlp2(X, 256, 512, W1, 1024, b1, W2, 512, b2, y))
    want = oracle.add(oracle.matmul(oracle.relu(oracle.add(oracle.matmul(X, W1), b1)), W2), b2)
    err = np.linalg.norm(y.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))
    assert err <= tol, err


def test_row_sums_honour_the_reduce_dims(rb):
    x = np.random.default_rng(2).uniform(-1, 1, (300, 777)).astype(np.float32)
    out = np.empty(300, np.float32)
    _ok(rb, rb.rb_row_sums(x, 300, 777, out))
    want = oracle.reduce(oracle.relu(x), (1,), f64=True)
    assert np.all(np.abs(out - want) <= 1e-5 * np.abs(want) + 1e-6)


def test_shape_error_reaches_the_caller(rb):
    a = np.ones((4, 5), np.float32)
    b = np.ones((4, 1), np.float32)
    assert rb.rb_bad_broadcast(a, 4, 5, b) != 0
    assert "Broadcasting addition not implemented" in rb.rb_last_error().decode()
