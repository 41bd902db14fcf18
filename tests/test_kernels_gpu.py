"""Parity of the sm_100a kernels with the CPU oracle, through the C-ABI.

Bounds (the reference CPU backend is the oracle, oracle/oracle.c):
  relu / add / multiply / transpose / split copies: bit-exact
  sigmoid: bit-exact against the reference formula 1/(1+expf(-x)) with this
           host's glibc expf (1 ulp on one float where the host's glibc is
           its build without FMA; oracle.sigmoid_ulp_bound())
  reductions: <= 1e-5 relative to the fp64 sum of the oracle's own
              element-wise values (the CPU's sequential fp32 sum is itself
              ~1e-4 off at 1e6 terms)
  matmul: norm-wise relative error <= 1e-5 (FFMA path), <= 2e-3 (TF32 path)
"""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

RTOL_REDUCE = 1e-5
RTOL_FFMA = 1e-5
RTOL_TF32 = 2e-3


def ulp_dist(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def normwise(got, want):
    want64 = want.astype(np.float64)
    return np.linalg.norm(got.astype(np.float64) - want64) / max(np.linalg.norm(want64), 1e-300)


def dev(ttc, a):
    return ttc.DeviceArray.from_numpy(a)


def run_unary(ttc, op, x):
    X = dev(ttc, x)
    Y = ttc.DeviceArray.empty(x.shape)
    rows = x.shape[0] if x.ndim > 1 else 1
    cols = x.size // rows
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(op), ttc.instr(ttc.OP_STORE, idx=0)]
    ttc.eltwise_chain(ttc.chain_desc(rows, cols, [ttc.in_view(X.ptr, cols)], [ttc.out_view(Y.ptr, cols)], prog))
    return Y.numpy()


SHAPES = [(1, 1), (1, 7), (3, 5), (64, 64), (1000, 1000), (17, 1028), (4099, 3)]


@pytest.mark.parametrize("shape", SHAPES)
def test_relu_bit_exact(ttc, shape):
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, shape).astype(np.float32)
    x.flat[0] = -0.0
    if x.size > 2:
        x.flat[1] = np.nan
        x.flat[2] = np.float32(1e-45)
    got = run_unary(ttc, ttc.OP_RELU, x)
    assert np.array_equal(got.view(np.int32), oracle.relu(x).view(np.int32))


def test_sigmoid_equals_reference_formula(ttc, golden):
    """README.md:332 formula 1.0f / (1.0f + std::exp(-x)), with this host's
    glibc expf: the kernel returns the same float (the device exp restates
    glibc's expf operation for operation), NaN, infinities and the slow path
    included; and the golden outputs recorded from the reference build."""
    rng = np.random.default_rng(1)
    bound = oracle.sigmoid_ulp_bound()
    specials = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 87.0, -87.0, 87.5, -87.5, 88.0, -88.0, 89.0, -89.0,
                         104.0, -104.0, 1e-45, -1e-45, 3.4e38, -3.4e38], np.float32)
    for x in (golden["sig_x"].reshape(1, -1), rng.uniform(-30, 30, (2048, 2048)).astype(np.float32),
              rng.uniform(-104, 89, (512, 1024)).astype(np.float32), specials.reshape(1, -1)):
        got = run_unary(ttc, ttc.OP_SIGMOID, x)
        want = oracle.sigmoid(x)
        assert np.array_equal(np.isnan(got), np.isnan(want))
        d = ulp_dist(got, want)
        d[np.isnan(want)] = 0
        assert d.max() <= bound and np.count_nonzero(d) <= bound, (d.max(), np.count_nonzero(d))
    got = run_unary(ttc, ttc.OP_SIGMOID, golden["sig_x"].reshape(1, -1))
    assert ulp_dist(got.ravel(), golden["sig_y"]).max() <= bound


def test_sigmoid_dense_sweep_equals_reference_formula(ttc):
    """Every 64th float of [-104, 104] (both signs, ~35M inputs), through the
    chain kernels: the same float as 1/(1+expf(-x)) on this host."""
    top = np.float32(104.0).view(np.int32)
    bits = np.arange(0, top, 64, dtype=np.int32)
    x = np.concatenate([bits.view(np.float32), (-bits.view(np.float32))])
    x = np.concatenate([x, np.zeros((-x.size) % 4096, np.float32)]).reshape(-1, 4096)
    got = run_unary(ttc, ttc.OP_SIGMOID, x)
    d = ulp_dist(got, oracle.sigmoid(x))
    assert d.max() <= oracle.sigmoid_ulp_bound()
    assert np.count_nonzero(d) <= oracle.sigmoid_ulp_bound()


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("op", ["add", "mul"])
def test_binary_bit_exact(ttc, shape, op):
    rng = np.random.default_rng(2)
    a = rng.uniform(-1, 1, shape).astype(np.float32)
    b = rng.uniform(-1, 1, shape).astype(np.float32)
    A, B = dev(ttc, a), dev(ttc, b)
    Y = ttc.DeviceArray.empty(shape)
    rows, cols = shape
    code = ttc.OP_ADD if op == "add" else ttc.OP_MUL
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(code, ttc.SRC_INPUT, 1), ttc.instr(ttc.OP_STORE, idx=0)]
    ttc.eltwise_chain(ttc.chain_desc(rows, cols, [ttc.in_view(A.ptr, cols), ttc.in_view(B.ptr, cols)],
                                     [ttc.out_view(Y.ptr, cols)], prog))
    want = oracle.add(a, b) if op == "add" else oracle.multiply(a, b)
    assert np.array_equal(Y.numpy(), want)


@pytest.mark.parametrize("shape", [(37, 64), (256, 1024), (5, 3), (300, 17)])
def test_bias_add_broadcast(ttc, shape, golden):
    rng = np.random.default_rng(3)
    a = rng.uniform(-1, 1, shape).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, (1, shape[1])).astype(np.float32)
    A, Bb = dev(ttc, a), dev(ttc, bias)
    Y = ttc.DeviceArray.empty(shape)
    rows, cols = shape
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_ADD, ttc.SRC_INPUT, 1), ttc.instr(ttc.OP_STORE, idx=0)]
    ttc.eltwise_chain(ttc.chain_desc(rows, cols, [ttc.in_view(A.ptr, cols), ttc.in_view(Bb.ptr, 0)],
                                     [ttc.out_view(Y.ptr, cols)], prog))
    assert np.array_equal(Y.numpy(), oracle.add(a, bias))


def test_readme_chain_fused_with_sum(ttc, golden):
    """w = multiply(add(relu(x), relu(x)), ...) and s = reduce_sum(w) in one kernel
    (the README chain, x[1000,1000] ~ U(-1,1))."""
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (1000, 1000)).astype(np.float32)
    X = dev(ttc, x)
    W = ttc.DeviceArray.empty(x.shape)
    S = ttc.DeviceArray.empty((1,))
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_RELU), ttc.instr(ttc.OP_ADD, ttc.SRC_ACC),
            ttc.instr(ttc.OP_MUL, ttc.SRC_ACC), ttc.instr(ttc.OP_STORE, idx=0)]
    ttc.eltwise_chain(ttc.chain_desc(1000, 1000, [ttc.in_view(X.ptr, 1000)], [ttc.out_view(W.ptr, 1000)], prog,
                                     reduce=ttc.REDUCE_ALL, reduce_out=S.ptr))
    y = oracle.relu(x)
    z = oracle.add(y, y)
    w = oracle.multiply(z, z)
    assert np.array_equal(W.numpy(), w)
    exact = oracle.reduce(w, f64=True)[0]
    s = S.numpy()[0]
    assert abs(s - exact) <= RTOL_REDUCE * abs(exact)
    # golden fixture of the lazy path (reference tape executor)
    c = golden["chain_x"]
    C_, Wc = dev(ttc, c), ttc.DeviceArray.empty(c.shape)
    ttc.eltwise_chain(ttc.chain_desc(c.shape[0], c.shape[1], [ttc.in_view(C_.ptr, c.shape[1])],
                                     [ttc.out_view(Wc.ptr, c.shape[1])], prog))
    assert np.array_equal(Wc.numpy(), golden["chain_w"])


@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (1000, 1000), (19, 300), (65, 4096), (4096, 20), (7, 2051)])
@pytest.mark.parametrize("mode", ["rows", "cols", "all"])
@pytest.mark.parametrize("mean", [False, True])
def test_chain_reductions(ttc, shape, mode, mean):
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, shape).astype(np.float32)
    X = dev(ttc, x)
    rows, cols = shape
    n_out = {"rows": rows, "cols": cols, "all": 1}[mode]
    red = {"rows": ttc.REDUCE_ROWS, "cols": ttc.REDUCE_COLS, "all": ttc.REDUCE_ALL}[mode]
    dims = {"rows": (1,), "cols": (0,), "all": ()}[mode]
    O = ttc.DeviceArray.empty((n_out,))
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_SIGMOID)]
    ttc.eltwise_chain(ttc.chain_desc(rows, cols, [ttc.in_view(X.ptr, cols)], [], prog, reduce=red,
                                     reduce_out=O.ptr, mean=mean))
    sig = oracle.sigmoid(x)
    want = oracle.reduce(sig, dims, mean=mean, f64=True).ravel()
    got = O.numpy()
    assert np.all(np.abs(got - want) <= RTOL_REDUCE * np.abs(want) + 1e-30), np.max(np.abs(got - want) / np.abs(want))


@pytest.mark.parametrize("shape,dims", [((1000,), ()), ((1000,), (0,)), ((19, 300), (1,)), ((19, 300), (0,)),
                                        ((4, 5, 6), (1,)), ((4, 5, 6), (0, 2)), ((3, 4, 5, 6), (1, 3)),
                                        ((3, 4, 5, 6), (0, 1, 2, 3)), ((3, 4, 5, 6), (-1,)), ((2, 3, 4, 5), (0, 3))])
@pytest.mark.parametrize("mean", [False, True])
def test_ttc_reduce_any_dims(ttc, shape, dims, mean):
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, shape).astype(np.float32)
    X = dev(ttc, x)
    want = oracle.reduce(x, dims, mean=mean, f64=True)
    O = ttc.DeviceArray.empty(want.shape)
    ttc.reduce(X.ptr, shape, dims, mean, O.ptr)
    got = O.numpy()
    assert np.allclose(got, want, rtol=RTOL_REDUCE, atol=1e-6)


def test_segments_and_column_broadcast(ttc):
    """8 segments (split chunks as views) of sigmoid(C) * relu(C + C), reduced
    along dim 1 of the transposed view: r_i[j] = sum_c f(A[2048 i + c, j])."""
    rng = np.random.default_rng(6)
    R, C, nseg = 64, 96, 8
    a = rng.uniform(-1, 1, (nseg * R, C)).astype(np.float32)
    A = dev(ttc, a)
    O = ttc.DeviceArray.empty((nseg, C))
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_ADD, ttc.SRC_ACC), ttc.instr(ttc.OP_RELU),
            ttc.instr(ttc.OP_SAVE, idx=0), ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_SIGMOID),
            ttc.instr(ttc.OP_MUL, ttc.SRC_SLOT, 0)]
    ttc.eltwise_chain(ttc.chain_desc(R, C, [ttc.in_view(A.ptr, C, 1, R * C)], [], prog, reduce=ttc.REDUCE_COLS,
                                     reduce_out=O.ptr, nseg=nseg, reduce_seg_stride=C))
    y = oracle.multiply(oracle.sigmoid(a), oracle.relu(oracle.add(a, a)))
    want = y.reshape(nseg, R, C).astype(np.float64).sum(axis=1)
    assert np.allclose(O.numpy(), want, rtol=RTOL_REDUCE, atol=1e-6)
    # column broadcast [R, 1] operand
    col = rng.uniform(-1, 1, (R, 1)).astype(np.float32)
    Cv = dev(ttc, col)
    Y = ttc.DeviceArray.empty((R, C))
    prog = [ttc.instr(ttc.OP_LOAD, idx=0), ttc.instr(ttc.OP_MUL, ttc.SRC_INPUT, 1), ttc.instr(ttc.OP_STORE, idx=0)]
    ttc.eltwise_chain(ttc.chain_desc(R, C, [ttc.in_view(A.ptr, C), ttc.in_view(Cv.ptr, 1, 0)],
                                     [ttc.out_view(Y.ptr, C)], prog))
    assert np.array_equal(Y.numpy(), (a[:R] * col).astype(np.float32))


@pytest.mark.parametrize("shape", [(1, 1), (23, 41), (64, 64), (1000, 1000), (129, 4097), (3, 16, 20)])
def test_transpose_bit_exact(ttc, shape):
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, shape).astype(np.float32)
    X = dev(ttc, x)
    out_shape = list(shape)
    out_shape[-1], out_shape[-2] = out_shape[-2], out_shape[-1]
    Y = ttc.DeviceArray.empty(out_shape)
    batch = int(np.prod(shape[:-2])) if len(shape) > 2 else 1
    ttc.transpose(X.ptr, Y.ptr, batch, shape[-2], shape[-1])
    assert np.array_equal(Y.numpy(), oracle.transpose(x))


@pytest.mark.parametrize("shape,split,dim", [((10,), 3, 0), ((12, 17), 5, 0), ((12, 17), 5, 1), ((64, 256), 32, 1)])
def test_split_chunks_as_strided_copies(ttc, shape, split, dim):
    rng = np.random.default_rng(8)
    x = rng.uniform(-1, 1, shape).astype(np.float32)
    X = dev(ttc, x)
    x2 = x.reshape(1, -1) if x.ndim == 1 else x
    d = 1 if x.ndim == 1 else dim
    for i, want in enumerate(oracle.split(x, split, dim)):
        w2 = want.reshape(1, -1) if want.ndim == 1 else want
        Y = ttc.DeviceArray.empty(w2.shape)
        off = i * split * (1 if d == 1 else x2.shape[1])
        ttc.copy2d(X.at(off), x2.shape[1], Y.ptr, w2.shape[1], w2.shape[0], w2.shape[1])
        assert np.array_equal(Y.numpy(), w2)


def _gemm_case(ttc, m, k, n, ta, tb, path, rng, act=None, bias=False):
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    a_st = np.ascontiguousarray(a.T) if ta else a
    b_st = np.ascontiguousarray(b.T) if tb else b
    A, B = dev(ttc, a_st), dev(ttc, b_st)
    Cd = ttc.DeviceArray.empty((m, n))
    epi = None
    bias_v = rng.uniform(-0.1, 0.1, (1, n)).astype(np.float32)
    if act or bias:
        Bv = dev(ttc, bias_v)
        prog, ins = [], []
        if bias:
            ins.append(ttc.in_view(Bv.ptr, 0))
            prog.append(ttc.instr(ttc.OP_ADD, ttc.SRC_INPUT, 0))
        if act == "relu":
            prog.append(ttc.instr(ttc.OP_RELU))
        if act == "sigmoid":
            prog.append(ttc.instr(ttc.OP_SIGMOID))
        prog.append(ttc.instr(ttc.OP_STORE, idx=0))
        epi = ttc.chain_desc(m, n, ins, [ttc.out_view(Cd.ptr, n)], prog)
    g = ttc.gemm(m, n, k, A.ptr, a_st.shape[1], B.ptr, b_st.shape[1], Cd.ptr, n, ta, tb, path, epi)
    want = oracle.matmul(a_st, b_st, ta, tb)
    if bias:
        want = oracle.add(want, bias_v)
    if act == "relu":
        want = oracle.relu(want)
    if act == "sigmoid":
        want = oracle.sigmoid(want)
    return Cd.numpy(), want, g


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (2, 2, 2), (45, 67, 29), (128, 128, 128), (256, 512, 1024),
                                   (257, 33, 130)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_ffma(ttc, m, k, n, ta, tb):
    rng = np.random.default_rng(9)
    got, want, _ = _gemm_case(ttc, m, k, n, ta, tb, ttc.GEMM_FFMA, rng)
    assert normwise(got, want) <= RTOL_FFMA


def test_gemm_known_answer(ttc):
    # tests/cpp/integration/test_end_to_end.cpp:58-89: 2s . 3s = 12
    A = dev(ttc, np.full((2, 2), 2, np.float32))
    B = dev(ttc, np.full((2, 2), 3, np.float32))
    C = ttc.DeviceArray.empty((2, 2))
    ttc.gemm(2, 2, 2, A.ptr, 2, B.ptr, 2, C.ptr, 2, path=ttc.GEMM_FFMA)
    assert np.all(C.numpy() == 12.0)


@pytest.mark.parametrize("m,k,n", [(128, 32, 256), (256, 512, 1024), (256, 1024, 512), (384, 100, 300),
                                   (1000, 260, 772), (128, 4096, 256), (520, 64, 1032), (1024, 512, 1280)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_tf32(ttc, m, k, n, ta, tb):
    rng = np.random.default_rng(10)
    got, want, g = _gemm_case(ttc, m, k, n, ta, tb, ttc.GEMM_TF32, rng)
    assert ttc.gemm_select_path(g) == ttc.GEMM_TF32
    err = normwise(got, want)
    assert err <= RTOL_TF32, err


@pytest.mark.parametrize("m,k,n", [(128, 32, 128), (256, 512, 1024), (384, 100, 300), (1000, 260, 772),
                                   (128, 4096, 256), (520, 64, 1032), (1024, 512, 1280)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_tf32x3(ttc, m, k, n, ta, tb):
    """Three-pass TF32 (x = big + small, big*big + big*small + small*big on
    the tensor cores): the FFMA path's 1e-5 bound."""
    rng = np.random.default_rng(16)
    got, want, g = _gemm_case(ttc, m, k, n, ta, tb, ttc.GEMM_TF32X3, rng, act="sigmoid", bias=True)
    assert ttc.gemm_select_path(g) == ttc.GEMM_TF32X3
    err = normwise(got, want)
    assert err <= RTOL_FFMA, err


def test_gemm_tf32x3_wide_range_and_small_shapes(ttc):
    """Operands spanning many binades keep the 1e-5 bound (the remainder is
    scaled with its element); shapes the tensor-core kernel does not take
    run on the FFMA path."""
    rng = np.random.default_rng(17)
    a = (rng.standard_normal((256, 384)) * np.exp2(rng.integers(-20, 20, (256, 384)))).astype(np.float32)
    b = (rng.standard_normal((384, 512)) * np.exp2(rng.integers(-20, 20, (384, 512)))).astype(np.float32)
    A, B = dev(ttc, a), dev(ttc, b)
    C = ttc.DeviceArray.empty((256, 512))
    ttc.gemm(256, 512, 384, A.ptr, 384, B.ptr, 512, C.ptr, 512, path=ttc.GEMM_TF32X3)
    assert normwise(C.numpy(), oracle.matmul(a, b)) <= RTOL_FFMA
    got, want, g = _gemm_case(ttc, 45, 67, 29, 0, 0, ttc.GEMM_TF32X3, rng)
    assert ttc.gemm_select_path(g) == ttc.GEMM_FFMA
    assert normwise(got, want) <= RTOL_FFMA


@pytest.mark.parametrize("m,k,n", [(256, 512, 1024), (256, 1024, 512), (200, 1000, 520), (128, 4096, 256)])
@pytest.mark.parametrize("act", ["relu", "sigmoid"])
def test_gemm_tf32_split_k(ttc, m, k, n, act, monkeypatch):
    """GEMMs with fewer output tiles than half the SMs split K over up to 16
    work items (raw partial tiles, then a fixed-order sum and the epilogue in
    a second kernel): the same bound against the oracle, close to the unsplit
    kernel, and bit-identical from run to run."""
    rng = np.random.default_rng(15)
    got, want, _ = _gemm_case(ttc, m, k, n, 0, 0, ttc.GEMM_TF32, rng, act=act, bias=True)
    assert normwise(got, want) <= RTOL_TF32
    again, _, _ = _gemm_case(ttc, m, k, n, 0, 0, ttc.GEMM_TF32, np.random.default_rng(15), act=act, bias=True)
    assert np.array_equal(got, again)
    monkeypatch.setenv("TTC_GEMM_SPLITK", "0")
    whole, _, _ = _gemm_case(ttc, m, k, n, 0, 0, ttc.GEMM_TF32, np.random.default_rng(15), act=act, bias=True)
    assert normwise(got, whole) <= RTOL_TF32


@pytest.mark.parametrize("path,m,n,k", [("tf32", 4096, 4096, 1024), ("tf32x3", 1664, 4864, 1024)])
def test_gemm_tail_wave_split(ttc, path, m, n, k, monkeypatch):
    """The opt-in split of a partly filled last wave (TTC_GEMM_TAILSPLIT=1;
    4096x4096: 512 tiles = 3 waves of 148 + 68, only those 68 tiles split
    along K): the same values as the unsplit launch up to fp32 summation
    order, the fused column sums too, and sampled rows (the last row block
    included) against the oracle. The single-CTA kernel is forced: the CTA-pair
    kernel, the default for this many tiles, does not split."""
    monkeypatch.setenv("TTC_GEMM_PAIR", "0")
    rng = np.random.default_rng(18)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, (1, n)).astype(np.float32)
    A, B, Bv = dev(ttc, a), dev(ttc, b), dev(ttc, bias)
    code = ttc.GEMM_TF32X3 if path == "tf32x3" else ttc.GEMM_TF32

    def run():
        C = ttc.DeviceArray.empty((m, n))
        S = ttc.DeviceArray.empty((n,))
        epi = ttc.chain_desc(m, n, [ttc.in_view(Bv.ptr, 0)], [ttc.out_view(C.ptr, n)],
                             [ttc.instr(ttc.OP_ADD, ttc.SRC_INPUT, 0), ttc.instr(ttc.OP_SIGMOID),
                              ttc.instr(ttc.OP_STORE, idx=0)], reduce=ttc.REDUCE_COLS, reduce_out=S.ptr)
        ttc.gemm(m, n, k, A.ptr, k, B.ptr, n, path=code, epilogue=epi)
        return C.numpy(), S.numpy()

    monkeypatch.setenv("TTC_GEMM_TAILSPLIT", "1")
    c1, s1 = run()
    monkeypatch.setenv("TTC_GEMM_TAILSPLIT", "0")
    c0, s0 = run()
    assert normwise(c1, c0) <= 1e-6 and normwise(s1, s0) <= 1e-6
    assert not np.array_equal(c1, c0) or path == "tf32x3"  # the split tiles sum in another order
    rows = np.concatenate([rng.choice(m - 128, 48, replace=False), np.arange(m - 16, m)])
    want = oracle.sigmoid(oracle.add(oracle.matmul(a[rows], b), bias))
    assert normwise(c1[rows], want) <= (RTOL_FFMA if path == "tf32x3" else RTOL_TF32)


@pytest.mark.parametrize("m,k,n", [(256, 512, 1024), (384, 100, 300), (1000, 260, 772), (520, 64, 1032),
                                   (1024, 512, 1280)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_gemm_tf32_cta_pair(ttc, m, k, n, ta, tb, monkeypatch):
    """The tcgen05.mma.cta_group::2 kernel (256x256 tile per CTA pair)."""
    monkeypatch.setenv("TTC_GEMM_PAIR", "1")
    rng = np.random.default_rng(13)
    got, want, _ = _gemm_case(ttc, m, k, n, ta, tb, ttc.GEMM_TF32, rng, act="sigmoid", bias=True)
    assert normwise(got, want) <= RTOL_TF32


@pytest.mark.parametrize("path", ["ffma", "tf32"])
@pytest.mark.parametrize("act", ["relu", "sigmoid", None])
def test_gemm_epilogue_fused_mlp(ttc, path, act, golden):
    """math::fused_mlp (fused_ops.cpp:39-61): bias then activation in the epilogue."""
    rng = np.random.default_rng(12)
    p = ttc.GEMM_FFMA if path == "ffma" else ttc.GEMM_TF32
    got, want, _ = _gemm_case(ttc, 256, 512, 1024, 0, 0, p, rng, act=act, bias=True)
    assert normwise(got, want) <= (RTOL_FFMA if path == "ffma" else RTOL_TF32)


def test_gemm_golden_fused_mlp(ttc, golden):
    x, w, b = golden["mm_a"], golden["mlp_w"], golden["mlp_b"]
    X, Wd, Bd = dev(ttc, x), dev(ttc, w), dev(ttc, b)
    Y = ttc.DeviceArray.empty((x.shape[0], w.shape[1]))
    epi = ttc.chain_desc(x.shape[0], w.shape[1], [ttc.in_view(Bd.ptr, 0)], [ttc.out_view(Y.ptr, w.shape[1])],
                         [ttc.instr(ttc.OP_ADD, ttc.SRC_INPUT, 0), ttc.instr(ttc.OP_RELU),
                          ttc.instr(ttc.OP_STORE, idx=0)])
    ttc.gemm(x.shape[0], w.shape[1], x.shape[1], X.ptr, x.shape[1], Wd.ptr, w.shape[1], path=ttc.GEMM_FFMA,
             epilogue=epi)
    assert normwise(Y.numpy(), golden["mlp_relu_y"]) <= RTOL_FFMA


def test_invalid_descriptors_are_errors(ttc):
    X = ttc.DeviceArray.empty((4, 4))
    bad = ttc.chain_desc(4, 4, [ttc.in_view(X.ptr, 4)], [], [ttc.instr(ttc.OP_RELU)])
    with pytest.raises(ttc.TTCError) as e:
        ttc.eltwise_chain(bad)
    assert e.value.code == ttc.ERR_INVALID
    bad = ttc.chain_desc(4, 4, [ttc.in_view(X.ptr, 4, 2)], [], [ttc.instr(ttc.OP_LOAD)])
    with pytest.raises(ttc.TTCError):
        ttc.eltwise_chain(bad)
    with pytest.raises(ttc.TTCError):
        ttc.gemm(4, 4, 4, X.ptr, 2, X.ptr, 4, X.ptr, 4)


@pytest.mark.parametrize("path", ["ffma", "tf32", "tf32_pair", "tf32x3"])
@pytest.mark.parametrize("m,k,n", [(256, 512, 1024), (1000, 260, 772), (520, 64, 1032), (200, 1000, 520)])
@pytest.mark.parametrize("mean,store", [(False, False), (True, True)])
def test_gemm_epilogue_column_sum(ttc, path, m, k, n, mean, store, monkeypatch):
    """Epilogue reduction TTC_REDUCE_COLS: the column sums (or means) over the
    M rows of the final epilogue value, from per-32-row partials written by
    the epilogue (TF32 kernels) or a column-sum chain (FFMA path); with STORE
    the matrix is written as well."""
    if path == "tf32_pair":
        monkeypatch.setenv("TTC_GEMM_PAIR", "1")
    rng = np.random.default_rng(14)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, (1, n)).astype(np.float32)
    A, B, Bv = dev(ttc, a), dev(ttc, b), dev(ttc, bias)
    S = ttc.DeviceArray.empty((n,))
    C = ttc.DeviceArray.empty((m, n))
    prog = [ttc.instr(ttc.OP_ADD, ttc.SRC_INPUT, 0), ttc.instr(ttc.OP_SIGMOID)]
    outs = []
    if store:
        prog.append(ttc.instr(ttc.OP_STORE, idx=0))
        outs = [ttc.out_view(C.ptr, n)]
    epi = ttc.chain_desc(m, n, [ttc.in_view(Bv.ptr, 0)], outs, prog, reduce=ttc.REDUCE_COLS, reduce_out=S.ptr,
                         mean=mean)
    p = {"ffma": ttc.GEMM_FFMA, "tf32x3": ttc.GEMM_TF32X3}.get(path, ttc.GEMM_TF32)
    ttc.gemm(m, n, k, A.ptr, k, B.ptr, n, path=p, epilogue=epi)
    y = oracle.sigmoid(oracle.add(oracle.matmul(a, b), bias))
    want = oracle.reduce(y, (0,), mean=mean, f64=True)
    tol = RTOL_FFMA if path in ("ffma", "tf32x3") else RTOL_TF32
    assert normwise(S.numpy(), want) <= tol
    if store:
        assert normwise(C.numpy(), y) <= tol


def test_gemm_epilogue_column_sum_of_no_rows(ttc):
    A = ttc.DeviceArray.empty((1, 8))
    B = ttc.DeviceArray.empty((8, 16))
    S = ttc.DeviceArray.empty((16,))
    for mean, want in ((False, 0.0), (True, np.nan)):
        epi = ttc.chain_desc(0, 16, [], [], [], reduce=ttc.REDUCE_COLS, reduce_out=S.ptr, mean=mean)
        ttc.gemm(0, 16, 8, A.ptr, 8, B.ptr, 16, epilogue=epi)
        got = S.numpy()
        assert np.all(np.isnan(got)) if mean else np.all(got == 0.0)
