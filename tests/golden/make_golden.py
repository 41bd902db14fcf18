"""Generates tests/golden/golden.npz from the reference's own code.

Run in a container where the reference sources are present:
    python tests/golden/make_golden.py
It builds oracle/_ref/libttref.so (oracle/build_ref.sh: the reference's
src/ compiled unmodified) and records seeded inputs with the reference's
outputs. The fixtures let the GPU tests and the CPU oracle tests check
parity where the reference sources are absent.

Sigmoid has no reference implementation (only the README recipe,
README.md:332); its fixture holds the C restatement's outputs (glibc expf).
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402


def main():
    oracle.build_ref()
    R = oracle.Ref()
    rng = np.random.default_rng(20240601)
    g = {}
    x = rng.uniform(-1, 1, (33, 70)).astype(np.float32)
    x[0, :4] = [0.0, -0.0, np.float32(1e-45), -np.float32(1e-45)]
    g["relu_x"], g["relu_y"] = x, R.relu(x)
    a = rng.uniform(-1, 1, (37, 64)).astype(np.float32)
    b = rng.uniform(-1, 1, (37, 64)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, (1, 64)).astype(np.float32)
    g["add_a"], g["add_b"], g["add_y"] = a, b, R.add(a, b)
    g["bias_b"], g["bias_y"] = bias, R.add(a, bias)
    g["mul_y"] = R.multiply(a, b)
    A = rng.standard_normal((45, 67)).astype(np.float32)
    B = rng.standard_normal((67, 29)).astype(np.float32)
    g["mm_a"], g["mm_b"], g["mm_y"] = A, B, R.matmul(A, B)
    g["mm_ta_y"] = R.matmul(np.ascontiguousarray(A.T), B, True, False)
    g["mm_tb_y"] = R.matmul(A, np.ascontiguousarray(B.T), False, True)
    g["mm_tatb_y"] = R.matmul(np.ascontiguousarray(A.T), np.ascontiguousarray(B.T), True, True)
    W = (rng.standard_normal((67, 48)) / np.sqrt(67)).astype(np.float32)
    bb = rng.uniform(-0.1, 0.1, (1, 48)).astype(np.float32)
    g["mlp_w"], g["mlp_b"] = W, bb
    g["mlp_relu_y"] = R.fused_mlp(A, W, bb, True)
    g["mlp_lin_y"] = R.fused_mlp(A, W, bb, False)
    r = rng.uniform(-1, 1, (19, 300)).astype(np.float32)
    g["rsum_x"], g["rsum_rows_y"] = r, R.reduce_sum(r, (1,))
    g["rsum_all_raw"] = R.reduce_sum(r, ())  # reference: input shape, sum in element 0
    t = rng.uniform(-1, 1, (23, 41)).astype(np.float32)
    g["tr_x"], g["tr_y"] = t, R.transpose(t)
    v = rng.uniform(-1, 1, (10,)).astype(np.float32)
    g["split_x"], g["split_y"] = v, R.split_1d(v, 3)
    c = rng.uniform(-1, 1, (1000, 8)).astype(np.float32)
    g["chain_x"], g["chain_w"] = c, R.lazy_chain(c)
    W1 = (rng.standard_normal((16, 24)) / 4).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, (1, 24)).astype(np.float32)
    W2 = (rng.standard_normal((24, 8)) / np.sqrt(24)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, (1, 8)).astype(np.float32)
    X = rng.standard_normal((12, 16)).astype(np.float32)
    g.update(mlp2_x=X, mlp2_w1=W1, mlp2_b1=b1, mlp2_w2=W2, mlp2_b2=b2, mlp2_y=R.lazy_mlp2(X, W1, b1, W2, b2))
    s = np.concatenate([rng.uniform(-20, 20, 4000), [0.0, -0.0, 88.0, -88.0, 104.0, -104.0]]).astype(np.float32)
    g["sig_x"], g["sig_y"] = s, oracle.sigmoid(s)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(out, **g)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
