"""End-to-end through the public front end (lazy graph -> tape -> fused
sm_100a kernels -> to_numpy), against the CPU oracle and the reference's own
known answers. Bounds as in test_kernels_gpu.py."""
import numpy as np
import pytest

import oracle
import tt_lazy_b200 as tl

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def fresh():
    tl.clear()
    tl.set_gemm_path("auto")
    yield
    tl.clear()


def normwise(got, want):
    w = want.astype(np.float64)
    return np.linalg.norm(got.astype(np.float64) - w) / max(np.linalg.norm(w), 1e-300)


def ulp_dist(a, b):
    a = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def test_reference_known_answers():
    # test_end_to_end.cpp:58-89
    r = tl.matmul(tl.constant(np.full((2, 2), 2, np.float32)), tl.constant(np.full((2, 2), 3, np.float32)))
    assert r.is_lazy
    assert np.all(r.numpy() == 12.0) and r.is_evaluated
    # test_end_to_end.cpp:94-124
    x = np.array([-2.0, -1.0, 0.0, 1.0, 2.0, -0.5, 0.5, -3.0], np.float32).reshape(2, 4)
    assert tl.relu(tl.constant(x)).numpy().ravel().tolist() == [0, 0, 0, 1, 2, 0, 0.5, 0]
    # test_mlp_demo.cpp:261-299
    two, three = tl.constant(np.full((2, 3), 2, np.float32)), tl.constant(np.full((2, 3), 3, np.float32))
    assert np.all(tl.add(two, three).numpy() == 5) and np.all(tl.multiply(two, three).numpy() == 6)


def test_materialized_inputs_work():
    # The reference drops materialized non-constant inputs (TapeGenerator.cpp:159-170).
    x = np.arange(-3, 3, dtype=np.float32).reshape(2, 3)
    assert np.array_equal(tl.relu(tl.materialized(x)).numpy(), oracle.relu(x))


def test_readme_chain_public_api(golden):
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (1000, 1000)).astype(np.float32)
    X = tl.constant(x)
    y = tl.relu(X)
    z = tl.add(y, y)
    w = tl.multiply(z, z)
    s = tl.reduce_sum(w)
    tl.evaluate([w, s])
    st = tl.stats()
    assert st["fused_operations"] == 1 and st["kernels_launched"] <= 3
    wn = w.numpy()
    ow = oracle.multiply(oracle.add(oracle.relu(x), oracle.relu(x)), oracle.add(oracle.relu(x), oracle.relu(x)))
    assert np.array_equal(wn, ow)
    exact = oracle.reduce(ow, f64=True)[0]
    assert abs(s.numpy()[0] - exact) <= 1e-5 * abs(exact)
    # the reference tape's own output (golden fixture)
    c = golden["chain_x"]
    C = tl.constant(c)
    yc = tl.relu(C)
    zc = tl.add(yc, yc)
    assert np.array_equal(tl.multiply(zc, zc).numpy(), golden["chain_w"])


@pytest.mark.parametrize("path,tol", [("ffma", 1e-5), ("tf32", 2e-3), ("tf32x3", 1e-5)])
def test_two_layer_mlp_mean(path, tol, golden):
    tl.set_gemm_path(path)
    rng = np.random.default_rng(1)
    X = rng.standard_normal((256, 512)).astype(np.float32)
    W1 = (rng.standard_normal((512, 1024)) / np.sqrt(512)).astype(np.float32)
    W2 = (rng.standard_normal((1024, 512)) / np.sqrt(1024)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, (1, 1024)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, (1, 512)).astype(np.float32)
    h = tl.relu(tl.add(tl.matmul(tl.constant(X), tl.constant(W1)), tl.constant(b1)))
    y = tl.add(tl.matmul(h, tl.constant(W2)), tl.constant(b2))
    m = tl.reduce_mean(y, [0])
    got_y, got_m = None, None
    tl.evaluate([y, m])
    got_y, got_m = y.numpy(), m.numpy()
    ho = oracle.relu(oracle.add(oracle.matmul(X, W1), b1))
    yo = oracle.add(oracle.matmul(ho, W2), b2)
    assert normwise(got_y, yo) <= tol
    mo = oracle.reduce(yo, (0,), mean=True, f64=True)
    assert normwise(got_m, mo) <= tol
    # the reference's lazy MLP (golden fixture) through the explicit path
    g = golden
    out = tl.add(tl.matmul(tl.relu(tl.add(tl.matmul(tl.constant(g["mlp2_x"]), tl.constant(g["mlp2_w1"])),
                                          tl.constant(g["mlp2_b1"]))), tl.constant(g["mlp2_w2"])),
                 tl.constant(g["mlp2_b2"]))
    assert normwise(out.numpy(), g["mlp2_y"]) <= tol


@pytest.mark.parametrize("has_relu", [True, False])
def test_explicit_fused_mlp(has_relu, golden):
    tl.set_gemm_path("ffma")
    g = golden
    y = tl.fused_mlp(tl.constant(g["mm_a"]), tl.constant(g["mlp_w"]), tl.constant(g["mlp_b"]), has_relu)
    want = g["mlp_relu_y"] if has_relu else g["mlp_lin_y"]
    assert normwise(y.numpy(), want) <= 1e-5


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 0), (0, 1), (1, 1)])
def test_matmul_transpose_flags(ta, tb):
    # handle_matmul in the reference drops transpose_a/b (OperationHandlers.cpp:61)
    tl.set_gemm_path("ffma")
    rng = np.random.default_rng(2)
    a = rng.standard_normal((40, 24)).astype(np.float32)
    b = rng.standard_normal((40, 24)).astype(np.float32) if (ta != tb) else rng.standard_normal((24, 40)).astype(np.float32)
    A = a if not ta else np.ascontiguousarray(a.T)
    B = b
    if ta == 0 and tb == 0:
        A, B = a, rng.standard_normal((24, 40)).astype(np.float32)
    elif ta == 1 and tb == 0:
        A, B = rng.standard_normal((24, 40)).astype(np.float32), rng.standard_normal((24, 32)).astype(np.float32)
    elif ta == 0 and tb == 1:
        A, B = rng.standard_normal((40, 24)).astype(np.float32), rng.standard_normal((32, 24)).astype(np.float32)
    else:
        A, B = rng.standard_normal((24, 40)).astype(np.float32), rng.standard_normal((32, 24)).astype(np.float32)
    got = tl.matmul(tl.constant(A), tl.constant(B), bool(ta), bool(tb)).numpy()
    assert normwise(got, oracle.matmul(A, B, ta, tb)) <= 1e-5


def test_transpose_split_views_feed_fused_chains():
    rng = np.random.default_rng(3)
    a = rng.uniform(-1, 1, (512, 512)).astype(np.float32)
    T = tl.transpose(tl.constant(a))
    chunks = tl.split(T, 64, 1)
    outs = [tl.reduce_sum(tl.multiply(tl.sigmoid(ch), tl.relu(tl.add(ch, ch))), [1]) for ch in chunks]
    tl.evaluate(outs)
    t = oracle.transpose(a)
    for i, o in enumerate(outs):
        ch = t[:, 64 * i:64 * (i + 1)]
        y = oracle.multiply(oracle.sigmoid(np.ascontiguousarray(ch)), oracle.relu(oracle.add(ch, ch)))
        want = oracle.reduce(y, (1,), f64=True)
        assert np.allclose(o.numpy(), want, rtol=1e-5, atol=1e-6)
    # materialising a transposed view and split chunks: bit-exact copies
    assert np.array_equal(tl.transpose(tl.constant(a)).numpy(), t)
    parts = tl.split(tl.constant(a), 100, 0)
    tl.evaluate(parts)
    for p, want in zip(parts, oracle.split(a, 100, 0)):
        assert np.array_equal(p.numpy(), want)
    cols = tl.split(tl.constant(a), 200, 1)
    for p, want in zip(cols, oracle.split(a, 200, 1)):
        assert np.array_equal(p.numpy(), want)


@pytest.mark.parametrize("transposed", [False, True])
def test_segmented_chains_match_per_chunk_oracle(transposed):
    # one segmented launch for the equal chunks; stored intermediates and the
    # per-chunk reductions of every segment are returned separately
    rng = np.random.default_rng(5)
    a = rng.uniform(-2, 2, (192, 160)).astype(np.float32)
    src = tl.transpose(tl.constant(a)) if transposed else tl.constant(a)
    base = oracle.transpose(a) if transposed else a
    chunks = tl.split(src, 48, 1)  # 160 or 192 columns: ragged last chunk when 160
    mids, reds = [], []
    for ch in chunks:
        m = tl.relu(tl.add(tl.sigmoid(ch), ch))
        mids.append(m)
        reds.append(tl.reduce_mean(tl.multiply(m, ch), [0]))
    tl.evaluate(mids + reds)
    for i, (m, r) in enumerate(zip(mids, reds)):
        ch = np.ascontiguousarray(base[:, 48 * i:48 * (i + 1)])
        mo = oracle.relu(oracle.add(oracle.sigmoid(ch), ch))
        assert m.shape == list(ch.shape)
        assert ulp_dist(m.numpy(), mo).max() <= oracle.sigmoid_ulp_bound()
        want = oracle.reduce(oracle.multiply(mo, ch), (0,), mean=True, f64=True)
        assert np.allclose(r.numpy(), want, rtol=1e-5, atol=1e-6)


def test_segmented_chain_on_strided_rank3_chunks_falls_back():
    # chunks of a middle-dim split are not addressable by (row, col) strides:
    # the segments then run one by one, with the same results
    rng = np.random.default_rng(6)
    a = rng.uniform(-1, 1, (4, 12, 8)).astype(np.float32)
    chunks = tl.split(tl.constant(a), 3, 1)
    outs = [tl.multiply(tl.relu(ch), ch) for ch in chunks]
    tl.evaluate(outs)
    for o, ch in zip(outs, oracle.split(a, 3, 1)):
        ch = np.ascontiguousarray(ch)
        assert np.array_equal(o.numpy(), oracle.multiply(oracle.relu(ch), ch))


@pytest.mark.parametrize("shape,dim,size", [((4, 12, 8), 2, 5), ((4, 12, 8), 0, 3), ((2, 3, 6, 8), 1, 2),
                                            ((2, 3, 6, 8), 3, 4), ((3, 5, 7), 1, 7)])
def test_rank3_and_rank4_views_materialise_bit_exact(shape, dim, size):
    # chunks of a transposed rank-3/4 tensor are strided windows of it;
    # reading them back and feeding them to a chain both densify on the device
    rng = np.random.default_rng(7)
    a = rng.uniform(-1, 1, shape).astype(np.float32)
    T = tl.transpose(tl.constant(a))
    t = oracle.transpose(a)
    chunks = tl.split(T, size, dim)
    relus = [tl.relu(ch) for ch in chunks]
    tl.evaluate(chunks + relus)
    want = oracle.split(t, size, dim)
    assert len(chunks) == len(want)
    for ch, r, w in zip(chunks, relus, want):
        w = np.ascontiguousarray(w)
        assert ch.shape == list(w.shape)
        assert np.array_equal(ch.numpy(), w)
        assert np.array_equal(r.numpy(), oracle.relu(w))


@pytest.mark.parametrize("dims,keep", [([], False), ([0], False), ([1], True), ([0, 1], False), ([-1], False)])
@pytest.mark.parametrize("mean", [False, True])
def test_reduce_semantics(dims, keep, mean):
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (37, 91)).astype(np.float32)
    op = tl.reduce_mean if mean else tl.reduce_sum
    r = op(tl.constant(x), dims, keep)
    want = oracle.reduce(x, tuple(dims), keepdim=keep, mean=mean, f64=True)
    assert r.shape == list(want.shape)
    assert np.allclose(r.numpy(), want, rtol=1e-5, atol=1e-6)


def test_cache_and_clear():
    x = tl.constant(np.ones((4, 4), np.float32))
    y = tl.relu(x)
    y.eval()
    h0 = tl.stats()["cache_hits"]
    z = tl.relu(x)
    tl.evaluate([z])
    tl.clear()
    # node ids restart after clear(); the cache must not return the old result
    x2 = tl.constant(-np.ones((4, 4), np.float32))
    assert np.all(tl.relu(x2).numpy() == 0)
    assert h0 >= 0


def test_random_dag_matches_oracle():
    """Small instance of the DCE / fusion stress graph: random ops over
    [64, 64], 40% of the nodes unreachable, reductions at the sinks."""
    tl.set_gemm_path("ffma")
    rng = np.random.default_rng(4)
    base = [rng.uniform(-0.5, 0.5, (64, 64)).astype(np.float32) for _ in range(4)]
    lazy = [tl.constant(b) for b in base]
    host = list(base)
    reach = []
    for i in range(60):
        k = int(rng.integers(0, 5))
        ia, ib = int(rng.integers(0, len(lazy))), int(rng.integers(0, len(lazy)))
        if k == 0:
            lazy.append(tl.relu(lazy[ia])); host.append(oracle.relu(host[ia]))
        elif k == 1:
            lazy.append(tl.sigmoid(lazy[ia])); host.append(oracle.sigmoid(host[ia]))
        elif k == 2:
            lazy.append(tl.add(lazy[ia], lazy[ib])); host.append(oracle.add(host[ia], host[ib]))
        elif k == 3:
            lazy.append(tl.multiply(lazy[ia], lazy[ib])); host.append(oracle.multiply(host[ia], host[ib]))
        else:
            lazy.append(tl.matmul(lazy[ia], lazy[ib])); host.append(oracle.matmul(host[ia], host[ib]))
    sinks = list(range(len(lazy) - 6, len(lazy)))
    outs = [tl.reduce_sum(lazy[s], [1]) for s in sinks]
    tl.evaluate(outs)
    for s, o in zip(sinks, outs):
        want = oracle.reduce(host[s], (1,), f64=True)
        scale = np.abs(host[s]).astype(np.float64).sum(axis=1) + 1e-30
        assert np.all(np.abs(o.numpy() - want) <= 1e-4 * scale)


def _matmul_depth(program, sinks):
    """Largest number of matmuls on any path from x0 to each sink value."""
    depth = [0]
    for kind, a, b in program:
        d = depth[a] + (kind == "matmul")
        if kind in ("add", "multiply") and not isinstance(b, str):
            d = max(d, depth[b])
        depth.append(d)
    return [depth[v] for v in sinks]


def _replay_rows(inputs, program, sinks, rows):
    """The stress program on rows `rows` of x0 and the gates, with the
    oracle's operations (every operation is row-local)."""
    need = set(sinks)
    for i in range(len(program), 0, -1):  # values the sinks read
        if i in need:
            kind, a, b = program[i - 1]
            need.add(a)
            if kind in ("add", "multiply") and not isinstance(b, str):
                need.add(b)
    gates = {g: np.ascontiguousarray(inputs[g][rows]) for g in ("g0", "g1")}
    vals = {0: np.ascontiguousarray(inputs["x0"][rows])}
    for i, (kind, a, b) in enumerate(program, start=1):
        if i not in need:
            continue
        if kind == "matmul":
            vals[i] = oracle.matmul(vals[a], inputs[b])
        elif kind == "relu":
            vals[i] = oracle.relu(vals[a])
        elif kind == "sigmoid":
            vals[i] = oracle.sigmoid(vals[a])
        elif kind == "add":
            vals[i] = oracle.add(vals[a], vals[b])
        else:
            vals[i] = oracle.multiply(vals[a], gates[b] if isinstance(b, str) else vals[b])
    return [vals[v] for v in sinks]


@pytest.mark.parametrize("path,per_matmul", [("tf32x3", 1e-5), ("auto", 2e-3)])
def test_dag_stress_at_full_size_on_sampled_rows(path, per_matmul):
    """The DCE / fusion stress graph at its benchmark size (seed 4: 200
    operations over [4096, 4096], 80 unreachable, reduce_sum(dim 1) at 4
    sinks). The unreachable operations never reach the tape. Every operation
    is row-local, so sampled rows of each sink are replayed on the oracle:
    the row sums must lie within the matmul path's norm-wise bound times the
    number of matmuls on the sink's longest path (1e-5 each for the
    fp32-accurate TF32X3 path, 2e-3 for TF32), relative to the row's sum of
    magnitudes, computed in fp64 over the oracle's own element values."""
    from tt_lazy_b200 import workloads

    tl.set_gemm_path(path)
    inputs, program, work = workloads.dag_stress_program()
    assert work["dead_ops"] == 80 and work["graph_nodes"] == 204
    outs = workloads.dag_build(inputs, program, work["sinks"])
    plan = tl.Plan(outs)
    assert len(plan) <= work["live_ops"]  # no unreachable operation is on the tape
    plan.run()
    got = [plan.numpy(i) for i in range(len(outs))]
    rows = [0, 1, 2047, 4095]
    want = _replay_rows(inputs, program, work["sinks"], rows)
    for g, w, depth in zip(got, want, _matmul_depth(program, work["sinks"])):
        exact = w.astype(np.float64).sum(axis=1)
        scale = np.abs(w).astype(np.float64).sum(axis=1)
        err = np.abs(g[rows].astype(np.float64) - exact) / scale
        assert err.max() <= max(depth, 1) * per_matmul, (path, depth, err.max())


@pytest.mark.parametrize("chunks", [2, 5])
def test_pipelined_plan_matches_the_whole_batch_plan(chunks):
    """Row chunks of a streamed batch, uploaded on the copy stream while
    earlier chunks compute, give the same column sums as one whole-batch
    evaluation (up to the order of the partial sums) and as the oracle."""
    tl.set_gemm_path("ffma")
    rng = np.random.default_rng(31)
    X = rng.standard_normal((1000, 128)).astype(np.float32)
    W1 = (rng.standard_normal((128, 256)) / np.sqrt(128)).astype(np.float32)
    W2 = (rng.standard_normal((256, 64)) / 16).astype(np.float32)
    xs = tl.streamed(X)
    s = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(xs, tl.constant(W1))), tl.constant(W2))), [0])
    whole, piped = tl.Plan([s]), tl.Plan([s], pipeline_chunks=chunks)
    whole.run()
    for _ in range(2):  # runs reuse the plan (and its device buffers)
        piped.run()
        got = piped.numpy(0)
        assert np.allclose(got, whole.numpy(0), rtol=1e-5, atol=1e-5)
    want = oracle.reduce(oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X, W1)), W2)), (0,), f64=True)
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)
    X[:] = rng.standard_normal(X.shape).astype(np.float32)  # a new batch in the same host buffer
    piped.run()
    want = oracle.reduce(oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X, W1)), W2)), (0,), f64=True)
    assert np.allclose(piped.numpy(0), want, rtol=1e-5, atol=1e-5)


def test_pipelined_plan_over_a_resident_batch_matches_the_whole_batch_plan():
    """A resident batch (a constant) in 3 row chunks, on the TF32 path with
    the CTA-pair GEMM where the chunk fills the GPU: the same column sums as
    the whole-batch plan (up to the order of the partial sums) and, within
    the TF32 bound, as the oracle."""
    tl.set_gemm_path("auto")
    rng = np.random.default_rng(32)
    # a 2048-row chunk times W1 has 8 x 10 256x256 tiles: the CTA-pair kernel
    X = rng.standard_normal((6144, 32)).astype(np.float32)
    W1 = (rng.standard_normal((32, 2560)) / np.sqrt(32)).astype(np.float32)
    W2 = (rng.standard_normal((2560, 64)) / np.sqrt(2560)).astype(np.float32)
    s = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(tl.constant(X), tl.constant(W1))),
                                           tl.constant(W2))), [0])
    whole, piped = tl.Plan([s]), tl.Plan([s], pipeline_chunks=3)
    whole.run()
    for _ in range(2):
        piped.run()
        got = piped.numpy(0)
        assert np.allclose(got, whole.numpy(0), rtol=1e-5, atol=0)
    want = oracle.reduce(oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X, W1)), W2)), (0,), f64=True)
    assert normwise(got, want) <= 2e-3


def test_large_mlp_at_full_size_on_sampled_rows():
    """The 65536 x 4096 -> 16384 -> 4096 MLP at its full size (TF32 tensor-core
    GEMMs, fused relu / sigmoid epilogues, batch column sums): sampled rows of
    Y against the oracle (rows are independent), s against the fp64 sum of the
    GPU's own Y, and the row-pipelined plan against the whole-batch plan."""
    rng = np.random.default_rng(2)
    M, K, N = 65536, 4096, 16384
    X = rng.standard_normal((M, K), dtype=np.float32)
    W1 = (rng.standard_normal((K, N), dtype=np.float32) / np.float32(np.sqrt(K)))
    W2 = (rng.standard_normal((N, K), dtype=np.float32) / np.float32(np.sqrt(N)))
    xs = tl.streamed(X)
    y = tl.sigmoid(tl.matmul(tl.relu(tl.matmul(xs, tl.constant(W1))), tl.constant(W2)))
    s = tl.reduce_sum(y, [0])
    tl.evaluate([y, s])
    Y, S = y.numpy(), s.numpy()
    rows = [0, 1, 4095, 4096, 32767, 40000, 65534, 65535]
    want = oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X[rows], W1)), W2))
    assert normwise(Y[rows], want) <= 2e-3
    exact = Y.astype(np.float64).sum(axis=0)
    assert np.max(np.abs(S - exact) / np.abs(exact)) <= 1e-5
    s2 = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(xs, tl.constant(W1))), tl.constant(W2))), [0])
    piped = tl.Plan([s2], pipeline_chunks=8)  # s itself is materialised by now
    piped.run()
    assert np.allclose(piped.numpy(0), S, rtol=1e-5, atol=0)


def test_bandwidth_graph_at_full_size_on_sampled_outputs():
    """A[16384, 16384]: transpose -> 8 column chunks -> sigmoid(C) * relu(C + C)
    -> row sums, one segmented launch; sampled outputs of every chunk against
    the fp64 sum of the oracle's element-wise values."""
    rng = np.random.default_rng(3)
    n, w = 16384, 2048
    A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    outs = [tl.reduce_sum(tl.multiply(tl.sigmoid(ch), tl.relu(tl.add(ch, ch))), [1])
            for ch in tl.split(tl.transpose(tl.constant(A)), w, 1)]
    tl.evaluate(outs)
    for i, o in enumerate(outs):
        got = o.numpy()
        assert got.shape == (n,)
        for j in (0, 1, 777, 8191, 16383):
            c = np.ascontiguousarray(A[w * i:w * (i + 1), j])  # row j of chunk i of the transpose
            y = oracle.multiply(oracle.sigmoid(c), oracle.relu(oracle.add(c, c)))
            exact = y.astype(np.float64).sum()
            assert abs(got[j] - exact) <= 1e-5 * max(abs(exact), 1e-30), (i, j, got[j], exact)


def test_empty_and_degenerate_shapes():
    """Empty batches, an empty contraction and a split larger than its dim,
    as the reference's math functions handle them (empty results; a sum over
    nothing is 0; one chunk)."""
    e = np.zeros((0, 8), np.float32)
    assert tl.relu(tl.constant(e)).numpy().shape == (0, 8)
    assert tl.add(tl.constant(e), tl.constant(e)).numpy().shape == (0, 8)
    assert tl.sigmoid(tl.constant(e)).numpy().shape == (0, 8)
    assert np.array_equal(tl.reduce_sum(tl.constant(e), [0]).numpy(), np.zeros(8, np.float32))
    assert tl.reduce_sum(tl.constant(e), [1]).numpy().shape == (0,)
    for path in ("ffma", "tf32"):
        tl.set_gemm_path(path)
        a = np.ones((0, 16), np.float32)
        assert tl.matmul(tl.constant(a), tl.constant(np.ones((16, 8), np.float32))).numpy().shape == (0, 8)
        z = tl.matmul(tl.constant(np.ones((4, 0), np.float32)), tl.constant(np.ones((0, 8), np.float32))).numpy()
        assert z.shape == (4, 8) and np.all(z == 0)
    x = np.arange(15, dtype=np.float32).reshape(5, 3)
    parts = tl.split(tl.constant(x), 10, 0)
    assert len(parts) == 1 and np.array_equal(parts[0].numpy(), x)


def test_captured_plan_replays_the_tape_as_one_graph():
    """Plan.capture(): one warm run, then the tape recorded into a CUDA graph;
    replays give the same bits as the uncaptured plan, and a streamed input
    is re-read from its host memory on every replay."""
    rng = np.random.default_rng(41)
    x = rng.uniform(-1, 1, (1000, 1000)).astype(np.float32)
    xs = tl.streamed(x)
    y = tl.relu(xs)
    z = tl.add(y, y)
    w = tl.multiply(z, z)
    s = tl.reduce_sum(w)
    plain, cap = tl.Plan([w, s]), tl.Plan([w, s])
    plain.run()
    cap.capture()
    assert cap.captured
    for _ in range(3):
        cap.run()
        assert np.array_equal(cap.numpy(0), plain.numpy(0))
        assert np.array_equal(cap.numpy(1), plain.numpy(1))
    x[:] = rng.uniform(-1, 1, x.shape).astype(np.float32)
    cap.run()
    ow = oracle.multiply(oracle.add(oracle.relu(x), oracle.relu(x)), oracle.add(oracle.relu(x), oracle.relu(x)))
    assert np.array_equal(cap.numpy(0), ow)
    exact = oracle.reduce(ow, f64=True)[0]
    assert abs(cap.numpy(1)[0] - exact) <= 1e-5 * abs(exact)


@pytest.mark.parametrize("path,tol", [("tf32", 2e-3), ("tf32x3", 1e-5)])
def test_captured_pipelined_mlp_plan(path, tol):
    """Row chunks of 512: the GEMMs have 8 and 4 output tiles, so they run
    split-K (and, on tf32x3, with the operand split) inside the graph."""
    tl.set_gemm_path(path)
    rng = np.random.default_rng(42)
    X = rng.standard_normal((2048, 256)).astype(np.float32)
    W1 = (rng.standard_normal((256, 512)) / 16).astype(np.float32)
    W2 = (rng.standard_normal((512, 256)) / np.sqrt(512)).astype(np.float32)
    xs = tl.streamed(X)
    s = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(xs, tl.constant(W1))), tl.constant(W2))), [0])
    plain, cap = tl.Plan([s], pipeline_chunks=4), tl.Plan([s], pipeline_chunks=4)
    plain.run()
    cap.capture()
    for _ in range(2):
        cap.run()
        assert np.array_equal(cap.numpy(0), plain.numpy(0))
    want = oracle.reduce(oracle.sigmoid(oracle.matmul(oracle.relu(oracle.matmul(X, W1)), W2)), (0,), f64=True)
    assert normwise(cap.numpy(0), want) <= tol
    with pytest.raises(RuntimeError, match="all-reduce"):
        tl.Plan([tl.all_reduce_sum(s)]).capture()


def test_profiling_times_every_tape_operation():
    """set_profiling(True): each tape operation runs between two CUDA-event
    marks inside an NVTX range named after it; profile() lists them in tape
    order with their device times."""
    rng = np.random.default_rng(43)
    X = rng.standard_normal((512, 256)).astype(np.float32)
    W1 = (rng.standard_normal((256, 512)) / 16).astype(np.float32)
    W2 = (rng.standard_normal((512, 128)) / np.sqrt(512)).astype(np.float32)
    s = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(tl.constant(X), tl.constant(W1))), tl.constant(W2))),
                      [0])
    names = [o["op"] for o in tl.tape([s])]
    tl.set_profiling(True)
    try:
        plan = tl.Plan([s])
        plan.run()
        prof = tl.profile()
    finally:
        tl.set_profiling(False)
    assert [p["op"] for p in prof] == names
    assert all(p["ms"] > 0 for p in prof)
    plan.capture()  # recording turns the marks off by itself
    plan.run()
    assert tl.profile() == prof or len(tl.profile()) == len(prof)


def test_guard_bands_find_no_overrun_and_catch_a_planted_one():
    """Canary mode: every device buffer carries a 256-byte guard band that is
    read back after each tape operation. The hot-path graphs (chains with
    ragged shapes, segmented chains over transposed views, TF32 / FFMA GEMMs
    with epilogue column sums, densified rank-3 views) leave every band
    intact; a band overwritten on purpose (an in-bounds host write into the
    band itself) is reported."""
    from tt_lazy_b200 import capi

    tl.set_canaries(True)
    try:
        rng = np.random.default_rng(44)
        x = rng.uniform(-1, 1, (999, 1001)).astype(np.float32)
        X = tl.constant(x)
        w = tl.multiply(tl.add(tl.relu(X), X), tl.sigmoid(X))
        tl.evaluate([w, tl.reduce_sum(w, [0]), tl.reduce_mean(w, [1])])
        a = rng.uniform(-1, 1, (192, 160)).astype(np.float32)
        outs = [tl.reduce_sum(tl.multiply(tl.sigmoid(c), tl.relu(tl.add(c, c))), [1])
                for c in tl.split(tl.transpose(tl.constant(a)), 48, 1)]
        tl.evaluate(outs)
        for path in ("tf32", "ffma"):
            tl.set_gemm_path(path)
            m = rng.standard_normal((520, 64)).astype(np.float32)
            k = (rng.standard_normal((64, 1032)) / 8).astype(np.float32)
            tl.evaluate([tl.reduce_sum(tl.sigmoid(tl.matmul(tl.constant(m), tl.constant(k))), [0])])
        r3 = rng.uniform(-1, 1, (4, 12, 8)).astype(np.float32)
        tl.evaluate([tl.relu(ch) for ch in tl.split(tl.transpose(tl.constant(r3)), 5, 2)])
        assert tl.check_canaries() == []
        # planted: overwrite a live result's guard band from the host
        plan = tl.Plan([tl.relu(tl.constant(x))])
        plan.run()
        ptr = plan.device_ptr(0)
        off = tl.canary_offset(ptr)
        assert off >= x.nbytes
        junk = np.zeros(64, np.float32)
        capi.check(capi.lib().ttc_memcpy_h2d(capi.C.c_void_p(ptr + off), junk.ctypes.data_as(capi.C.c_void_p), 256))
        bad = tl.check_canaries()
        assert len(bad) == 1 and "overwritten" in bad[0]
        band = np.frombuffer(bytes(0xA5 ^ i for i in range(256)), np.uint8).copy()  # put the band back
        capi.check(capi.lib().ttc_memcpy_h2d(capi.C.c_void_p(ptr + off), band.ctypes.data_as(capi.C.c_void_p), 256))
        assert tl.check_canaries() == []
    finally:
        tl.set_canaries(False)
        tl.set_gemm_path("auto")


SPECIALS = np.array([0.0, -0.0, 1e-45, -1e-45, 1.1754944e-38, -1.1754944e-38, 1.0, -1.0, 3.4028235e38,
                     -3.4028235e38, np.inf, -np.inf, np.nan, 88.7, -88.7, 104.0, -104.0, 1e30, -1e30, 0.5],
                    np.float32)


def _same_bits_or_both_nan(got, want):
    both_nan = np.isnan(got) & np.isnan(want)
    return np.all(both_nan | (got.view(np.int32) == want.view(np.int32)))


@pytest.mark.parametrize("shape", [(16, 64), (1024, 1024)])
def test_special_values_through_fused_chains(shape):
    """Zeros of both signs, subnormals, the float limits, infinities and NaN
    through relu / add / multiply (bit-exact, NaN where the reference gives
    NaN) and sigmoid (the reference formula's float): the small shape runs on
    the interpreting kernels, the large one on the program-specialised ones."""
    rng = np.random.default_rng(21)
    x = rng.uniform(-2, 2, shape).astype(np.float32)
    y = rng.uniform(-2, 2, shape).astype(np.float32)
    for i in range(0, x.size, 97):
        x.flat[i] = SPECIALS[(i // 97) % SPECIALS.size]
        y.flat[i] = SPECIALS[(i // 97 + 7) % SPECIALS.size]
    X, Y = tl.constant(x), tl.constant(y)
    r = tl.relu(X)
    chain = tl.multiply(tl.add(r, Y), tl.add(r, Y))
    tl.evaluate([chain])
    assert _same_bits_or_both_nan(chain.numpy(), oracle.multiply(oracle.add(oracle.relu(x), y),
                                                               oracle.add(oracle.relu(x), y)))
    s = tl.sigmoid(X)
    got = s.numpy()
    want = oracle.sigmoid(x)
    fin = ~np.isnan(want)
    assert np.all(np.isnan(got[~fin]))
    assert ulp_dist(got[fin], want[fin]).max() <= oracle.sigmoid_ulp_bound()
    assert np.all(got[x == np.inf] == 1.0) and np.all(got[x == -np.inf] == 0.0)
    seg = tl.multiply(tl.sigmoid(X), tl.relu(tl.add(X, X)))
    want = oracle.multiply(oracle.sigmoid(x), oracle.relu(oracle.add(x, x)))
    got = seg.numpy()
    assert np.all(np.isnan(got) == np.isnan(want))
    fin = ~np.isnan(want)
    assert ulp_dist(got[fin], want[fin]).max() <= oracle.sigmoid_ulp_bound()


@pytest.mark.parametrize("path", ["ffma", "tf32", "tf32x3"])
def test_gemm_propagates_infinities_and_nan(path):
    """A row of A holding +inf, another holding NaN: the product's rows are
    +-inf / NaN exactly where the reference's fp32 matmul has them (inf * 0
    gives NaN), the other rows stay finite and within the path's bound. On
    tf32x3 the 128-row block holding them takes the TF32 product alone
    (2e-3), the other row block keeps the 1e-5 bound."""
    tl.set_gemm_path(path)
    rng = np.random.default_rng(22)
    a = rng.standard_normal((256, 128)).astype(np.float32)
    b = (rng.standard_normal((128, 256)) / 12).astype(np.float32)
    b[5, :7] = 0.0
    a[3, 5] = np.inf
    a[9, 17] = np.nan
    got = tl.matmul(tl.constant(a), tl.constant(b)).numpy()
    want = oracle.matmul(a, b)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(np.isposinf(got), np.isposinf(want)) and np.array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    tol = 1e-5 if path == "ffma" else 2e-3
    assert normwise(got[fin], want[fin]) <= tol
    if path == "tf32x3":
        assert normwise(got[128:], want[128:]) <= 1e-5
    tl.set_gemm_path("auto")
