"""The CPU oracle (oracle/oracle.c) pinned against the reference.

* golden.npz: outputs of the reference's own code (oracle/_ref, built from
  its sources by tests/golden/make_golden.py) -- checked bit-exactly.
* known answers copied from the reference's tests (cited per test).
* when oracle/_ref is present, random shapes against the live reference.
"""
import numpy as np
import pytest

import oracle


def test_golden_bit_exact(golden):
    g = golden
    assert np.array_equal(oracle.relu(g["relu_x"]), g["relu_y"])
    assert np.array_equal(oracle.add(g["add_a"], g["add_b"]), g["add_y"])
    assert np.array_equal(oracle.add(g["add_a"], g["bias_b"]), g["bias_y"])
    assert np.array_equal(oracle.multiply(g["add_a"], g["add_b"]), g["mul_y"])
    A, B = g["mm_a"], g["mm_b"]
    assert np.array_equal(oracle.matmul(A, B), g["mm_y"])
    assert np.array_equal(oracle.matmul(np.ascontiguousarray(A.T), B, True, False), g["mm_ta_y"])
    assert np.array_equal(oracle.matmul(A, np.ascontiguousarray(B.T), False, True), g["mm_tb_y"])
    assert np.array_equal(oracle.matmul(np.ascontiguousarray(A.T), np.ascontiguousarray(B.T), True, True),
                          g["mm_tatb_y"])
    assert np.array_equal(oracle.fused_mlp(A, g["mlp_w"], g["mlp_b"], True), g["mlp_relu_y"])
    assert np.array_equal(oracle.fused_mlp(A, g["mlp_w"], g["mlp_b"], False), g["mlp_lin_y"])
    assert np.array_equal(oracle.reduce_sum(g["rsum_x"], (1,)), g["rsum_rows_y"])
    # reference reduce_sum(dims={}): input-shaped result, total in element 0
    # (reduce_sum.cpp:28-32 with the shape rule of reduce_sum.cpp:12-18).
    raw = g["rsum_all_raw"]
    assert raw.size == g["rsum_x"].size and np.all(raw[1:] == 0)
    assert oracle.reduce_sum(g["rsum_x"])[0] == raw[0]
    assert np.array_equal(oracle.transpose(g["tr_x"]), g["tr_y"])
    assert np.array_equal(np.concatenate(oracle.split(g["split_x"], 3)), g["split_y"])
    y = oracle.relu(g["chain_x"])
    z = oracle.add(y, y)
    assert np.array_equal(oracle.multiply(z, z), g["chain_w"])
    h = oracle.relu(oracle.add(oracle.matmul(g["mlp2_x"], g["mlp2_w1"]), g["mlp2_b1"]))
    assert np.array_equal(oracle.add(oracle.matmul(h, g["mlp2_w2"]), g["mlp2_b2"]), g["mlp2_y"])
    assert np.array_equal(oracle.sigmoid(g["sig_x"]), g["sig_y"])


def test_known_answers_from_reference_tests():
    # tests/cpp/integration/test_end_to_end.cpp:58-89: 2x2 of 2.0 times 2x2 of 3.0 = 12.0
    assert np.all(oracle.matmul(np.full((2, 2), 2, np.float32), np.full((2, 2), 3, np.float32)) == 12.0)
    # test_end_to_end.cpp:98,120: relu of the 8-vector
    x = np.array([-2.0, -1.0, 0.0, 1.0, 2.0, -0.5, 0.5, -3.0], np.float32).reshape(2, 4)
    assert oracle.relu(x).ravel().tolist() == [0.0, 0.0, 0.0, 1.0, 2.0, 0.0, 0.5, 0.0]
    # tests/cpp/benchmarks/test_mlp_demo.cpp:265-296: 2 + 3 = 5, 2 * 3 = 6
    two, three = np.full((2, 3), 2, np.float32), np.full((2, 3), 3, np.float32)
    assert np.all(oracle.add(two, three) == 5) and np.all(oracle.multiply(two, three) == 6)
    # tests/cpp/unit/math/test_math_ops.cpp:36-110 (printed values)
    assert oracle.relu(np.array([-2, -1, 0, 3], np.float32)).tolist() == [0, 0, 0, 3]
    assert oracle.reduce_sum(np.array([1, 2, 3], np.float32), (0,)).tolist() == [6]
    e = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    f = np.arange(1, 7, dtype=np.float32).reshape(3, 2)
    assert oracle.matmul(e, f).tolist() == [[22, 28], [49, 64]]
    g = np.array([1, 2, 3], np.float32)
    h = np.array([2, 3, 4], np.float32)
    assert oracle.add(g, h).tolist() == [3, 5, 7] and oracle.multiply(g, h).tolist() == [2, 6, 12]


def test_fused_mlp_demo_weights():
    # test_mlp_demo.cpp:16-60 deterministic SimpleMLP weights and input (63-79);
    # relu output is non-negative (test_mlp_demo.cpp:381).
    w1 = np.array([0.1 * (1 + 0.1 * (i % 10)) for i in range(32)], np.float32).reshape(4, 8)
    b1 = np.array([0.01 * (1 + 0.1 * (i % 10)) for i in range(8)], np.float32).reshape(1, 8)
    x = np.array([1.0, 0.5, -0.2, 0.8, -0.5, 1.2, 0.3, -0.1], np.float32).reshape(2, 4)
    y = oracle.fused_mlp(x, w1, b1, True)
    assert np.all(y >= 0) and np.all(np.isfinite(y))
    unfused = oracle.relu(oracle.add(oracle.matmul(x, w1), b1))
    assert np.array_equal(y, unfused)


def test_shape_errors_mirror_reference():
    a = np.ones((4, 5), np.float32)
    with pytest.raises(oracle.OracleError, match="Broadcasting addition not implemented"):
        oracle.add(a, np.ones((4, 1), np.float32))
    with pytest.raises(oracle.OracleError, match="Broadcasting multiplication not fully implemented"):
        oracle.multiply(a, np.ones((1, 5), np.float32))
    with pytest.raises(oracle.OracleError, match="dimension mismatch"):
        oracle.matmul(a, a)
    with pytest.raises(oracle.OracleError, match="Split size must be positive"):
        oracle.split(a, 0)


def test_reduce_general_dims():
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, (3, 4, 5, 6)).astype(np.float32)
    for dims in [(0,), (1,), (2,), (3,), (0, 2), (1, 3), (0, 1, 2, 3), (1, 2)]:
        want = x.astype(np.float64).sum(axis=dims)
        got = oracle.reduce(x, dims, f64=True)
        assert np.allclose(got, want.reshape(got.shape), rtol=1e-12, atol=1e-12)
        assert np.allclose(oracle.reduce(x, dims), want.reshape(got.shape), rtol=1e-5, atol=1e-5)
        m = oracle.reduce(x, dims, mean=True)
        assert np.allclose(m, (want / np.prod([x.shape[d] for d in dims])).reshape(m.shape), atol=1e-6)


ref_missing = oracle.ref() is None


@pytest.mark.skipif(ref_missing, reason="oracle/_ref not built (reference sources absent)")
def test_against_live_reference():
    R = oracle.Ref()
    rng = np.random.default_rng(11)
    for shape in [(1, 1), (7, 13), (64, 100), (3, 1025)]:
        x = rng.uniform(-2, 2, shape).astype(np.float32)
        y = rng.uniform(-2, 2, shape).astype(np.float32)
        assert np.array_equal(oracle.relu(x), R.relu(x))
        assert np.array_equal(oracle.add(x, y), R.add(x, y))
        assert np.array_equal(oracle.multiply(x, y), R.multiply(x, y))
        bias = rng.uniform(-1, 1, (1, shape[1])).astype(np.float32)
        assert np.array_equal(oracle.add(x, bias), R.add(x, bias))
        assert np.array_equal(oracle.transpose(x), R.transpose(x))
        assert np.array_equal(oracle.reduce_sum(x, (1,)), R.reduce_sum(x, (1,)))
        assert oracle.reduce_sum(x)[0] == R.reduce_sum(x)[0]
    for m, k, n in [(1, 1, 1), (5, 9, 3), (33, 65, 17)]:
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        assert np.array_equal(oracle.matmul(a, b), R.matmul(a, b))
        bb = rng.uniform(-1, 1, (1, n)).astype(np.float32)
        assert np.array_equal(oracle.fused_mlp(a, b, bb, True), R.fused_mlp(a, b, bb, True))
    x = rng.uniform(-1, 1, (50, 16)).astype(np.float32)
    y = oracle.relu(x)
    z = oracle.add(y, y)
    assert np.array_equal(R.lazy_chain(x), oracle.multiply(z, z))


def test_expf_restatement_pinned_to_libm():
    """oracle.expf_ref (glibc's expf as its FMA build computes it) against this
    process's expf on every 61st bit pattern and the specials; on a host whose
    glibc picks that build they agree everywhere (the host test of the device
    header checks all 2^32 floats)."""
    u = np.arange(0, 1 << 32, 61, dtype=np.uint64).astype(np.uint32)
    x = np.concatenate([u.view(np.float32), np.array([np.inf, -np.inf, np.nan, 88.0, -88.0] + [float.fromhex(h) for h in (
        "0x1.62e42ep6", "-0x1.9fe368p6", "0x1.04845ep+5", "-0x1.f8cbb2p+5")], np.float32)])
    a, b = oracle.expf_ref(x), oracle.expf_libm(x)
    diff = (a.view(np.int32) != b.view(np.int32)) & ~(np.isnan(a) & np.isnan(b))
    if oracle.expf_is_fma_build():
        assert not diff.any(), x[diff][:8]
    else:
        assert diff.sum() <= 2
    # the reference formula through libm equals the restatement's sigmoid
    xs = x[np.abs(x) < 200]
    want = (np.float32(1) / (np.float32(1) + oracle.expf_ref(-xs))).astype(np.float32)
    got = oracle.sigmoid(xs)
    assert np.sum(got.view(np.int32) != want.view(np.int32)) <= oracle.sigmoid_ulp_bound()
