"""Front end on the CPU: graph building, shapes and errors (the reference's
graph-only unit / integration tests, tests/cpp/unit/*, tests/cpp/integration/
test_operations.cpp), tape generation, dead-code elimination and what the
fusion passes make of each workload's graph. Nothing here evaluates."""
import numpy as np
import pytest

import tt_lazy_b200 as tl


@pytest.fixture(autouse=True)
def fresh():
    tl.clear()
    yield
    tl.clear()


def c(shape, seed=0):
    return tl.constant(np.random.default_rng(seed).uniform(-1, 1, shape).astype(np.float32))


def test_lazy_shapes_keep_true_rank():
    x = c((2, 4))
    y = tl.relu(x)
    assert y.is_lazy and not y.is_evaluated
    assert y.shape == [2, 4] and y.rank == 2
    assert tl.matmul(x, c((4, 3))).shape == [2, 3]
    assert tl.matmul(x, c((2, 3)), transpose_a=True).shape == [4, 3]
    assert tl.transpose(x).shape == [4, 2]
    assert tl.reduce_sum(x).shape == [1]
    assert tl.reduce_sum(x, [1]).shape == [2]
    assert tl.reduce_mean(x, [0], True).shape == [1, 4]
    parts = tl.split(c((10, 3)), 4, 0)
    assert [p.shape for p in parts] == [[4, 3], [4, 3], [2, 3]]
    assert [p.output_index for p in parts] == [0, 1, 2]
    assert tl.add(c((3, 5)), c((1, 5))).shape == [3, 5]
    assert tl.fused_mlp(x, c((4, 8)), c((1, 8))).shape == [2, 8]


def test_shape_errors_carry_reference_messages():
    with pytest.raises(RuntimeError, match="Broadcasting addition not implemented"):
        tl.add(c((3, 5)), c((3, 1)))
    with pytest.raises(RuntimeError, match="Broadcasting multiplication not fully implemented"):
        tl.multiply(c((3, 5)), c((1, 5)))
    with pytest.raises(RuntimeError, match="Matrix dimension mismatch"):
        tl.matmul(c((3, 5)), c((3, 5)))
    with pytest.raises(RuntimeError, match="Split size must be positive"):
        tl.split(c((4,)), 0)
    with pytest.raises(RuntimeError, match="Transpose requires at least 2D"):
        tl.transpose(c((4,)))


def ops(outs):
    return [o["op"] for o in tl.tape(outs)]


def test_readme_chain_fuses_to_one_kernel_with_tail_sum():
    x = c((1000, 1000))
    y = tl.relu(x)
    z = tl.add(y, y)
    w = tl.multiply(z, z)
    s = tl.reduce_sum(w)
    t = tl.tape([w, s])
    assert len(t) == 1
    assert t[0]["op"] == "FusedChain[relu -> add -> multiply -> reduce]"
    assert sorted(t[0]["outputs"]) == sorted([w.producer_node, s.producer_node])


def test_mlp_fusion_absorbs_bias_and_activation():
    X, W1, b1, W2, b2 = c((256, 512)), c((512, 1024)), c((1, 1024)), c((1024, 512)), c((1, 512))
    h = tl.relu(tl.add(tl.matmul(X, W1), b1))
    y = tl.add(tl.matmul(h, W2), b2)
    m = tl.reduce_mean(y, [0])
    # the batch-dim mean becomes the second GEMM's epilogue column sum
    assert ops([m]) == ["FusedGemm[matmul -> add -> relu]", "FusedGemm[matmul -> add -> reduce]"]
    # an intermediate requested as an output is not absorbed
    assert ops([m, h]) == ["FusedGemm[matmul -> add -> relu]", "FusedGemm[matmul -> add -> reduce]"]
    assert ops([m, y]) == ["FusedGemm[matmul -> add -> relu]", "FusedGemm[matmul -> add]", "Reduce"]
    tl.set_optimization(False)
    try:
        assert ops([m]) == ["MatMul", "Add", "ReLU", "MatMul", "Add", "Reduce"]
    finally:
        tl.set_optimization(True)


def test_large_mlp_sigmoid_then_batch_sum():
    X, W1, W2 = c((64, 32)), c((32, 128)), c((128, 32))
    y = tl.sigmoid(tl.matmul(tl.relu(tl.matmul(X, W1)), W2))
    s = tl.reduce_sum(y, [0])
    assert ops([s]) == ["FusedGemm[matmul -> relu]", "FusedGemm[matmul -> sigmoid -> reduce]"]
    # a reduction over the other dim is not a column sum: it stays a chain
    r = tl.reduce_sum(y, [1])
    assert ops([r]) == ["FusedGemm[matmul -> relu]", "FusedGemm[matmul -> sigmoid]", "Reduce"]


def test_bandwidth_graph_views_and_chains():
    A = c((64, 64))
    T = tl.transpose(A)
    chunks = tl.split(T, 8, 1)
    outs = []
    for ch in chunks:
        y = tl.multiply(tl.sigmoid(ch), tl.relu(tl.add(ch, ch)))
        outs.append(tl.reduce_sum(y, [1]))
    t = ops(outs)
    assert t == ["Transpose", "Split", "FusedChain[sigmoid -> add -> relu -> multiply -> reduce x8 segments]"]


def test_segment_fusion_needs_consecutive_equal_chunks():
    A = c((64, 48))
    chunks = tl.split(A, 20, 0)  # 20, 20, 20, 4: the ragged last chunk runs alone
    outs = [tl.reduce_sum(tl.relu(ch), [1]) for ch in chunks]
    t = ops(outs)
    assert t == ["Split", "FusedChain[relu -> reduce x3 segments]", "FusedChain[relu -> reduce]"]
    # different programs per chunk do not merge
    B = c((64, 48), 1)
    ch = tl.split(B, 16, 0)
    outs = [tl.relu(ch[0]), tl.sigmoid(ch[1]), tl.relu(ch[2]), tl.relu(ch[3])]
    t = ops(outs)
    assert t.count("FusedChain[relu x2 segments]") == 1 and "FusedChain[sigmoid]" in t


def test_dead_code_is_not_on_the_tape():
    x = c((8, 8))
    live = tl.relu(x)
    for _ in range(5):
        tl.sigmoid(tl.add(x, x))  # unreachable from `live`
    assert tl.graph_size() == 11
    t = tl.tape([live])
    assert len(t) == 1 and t[0]["op"].startswith("FusedChain[relu")


def test_random_dag_fusion_is_acyclic_and_complete():
    rng = np.random.default_rng(4)
    vals = [c((16, 16), i) for i in range(4)]
    nodes = []
    for i in range(120):
        kind = rng.integers(0, 5)
        a = vals[rng.integers(0, len(vals))]
        b = vals[rng.integers(0, len(vals))]
        v = [tl.relu, tl.sigmoid][kind % 2](a) if kind < 2 else \
            [tl.add, tl.multiply, lambda p, q: tl.matmul(p, q)][kind - 2](a, b)
        vals.append(v)
        nodes.append(v)
    outs = [tl.reduce_sum(v) for v in nodes[-5:]]
    t = tl.tape(outs)
    produced = set()
    for op in t:
        for i in op["inputs"]:
            assert i in produced, "operation reads a result produced later"
        produced.update(op["outputs"])
        produced.add(op["node"])


def test_pipelined_plan_rebuilds_the_graph_over_row_chunks():
    X = np.random.default_rng(0).standard_normal((64, 16)).astype(np.float32)
    xs = tl.streamed(X)
    W1, W2 = c((16, 32), 1), c((32, 8), 2)
    s = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(xs, W1)), W2)), [0])
    assert ops([s]) == ["FusedGemm[matmul -> relu]", "FusedGemm[matmul -> sigmoid -> reduce]"]
    assert len(tl.Plan([s])) == 2
    # 4 chunks x (GEMM, GEMM with the partial column sum) + the chunk-order sum of the partials (one chain)
    assert len(tl.Plan([s], pipeline_chunks=4)) == 9
    # the all-reduce runs once, after the partial sums are combined
    assert len(tl.Plan([tl.all_reduce_sum(s)], pipeline_chunks=3)) == 8
    # a streamed first chunk of 4096 rows or more is cut into 1/8, 1/8, 1/4 and 1/2 of it
    # (5 row ranges here); a resident batch is not (no upload to wait for)
    big = np.zeros((8192, 16), np.float32)
    for x, n_ops in ((tl.streamed(big), 11), (tl.constant(big), 5)):
        sb = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(x, W1)), W2)), [0])
        assert len(tl.Plan([sb], pipeline_chunks=2)) == n_ops


def test_pipelined_plan_over_a_resident_batch():
    """With no streamed input, the batch is the one resident rank-2 constant
    that is the matmuls' left operand; it is cut into constant row views (the
    same tape shape as a streamed batch). Two such constants are ambiguous."""
    xc = c((64, 16), 4)
    W1, W2 = c((16, 32), 1), c((32, 8), 2)
    s = tl.reduce_sum(tl.sigmoid(tl.matmul(tl.relu(tl.matmul(xc, W1)), W2)), [0])
    assert len(tl.Plan([s], pipeline_chunks=4)) == 9
    two = tl.reduce_sum(tl.add(tl.matmul(c((8, 16), 5), W1), tl.matmul(c((8, 16), 6), W1)), [0])
    with pytest.raises(RuntimeError, match="streamed rank-2 batch input"):
        tl.Plan([two], pipeline_chunks=2)
    # a materialized tensor owns its storage, which the plan's row views would not keep alive
    xm = tl.materialized(np.ones((64, 16), np.float32))
    with pytest.raises(RuntimeError, match="streamed rank-2 batch input"):
        tl.Plan([tl.reduce_sum(tl.matmul(xm, W1), [0])], pipeline_chunks=2)


def test_pipelined_plan_rejects_graphs_that_are_not_row_local():
    X = np.random.default_rng(0).standard_normal((64, 16)).astype(np.float32)
    xs = tl.streamed(X)
    bad = {
        "Transpose is not row-local": tl.reduce_sum(tl.transpose(xs), [0]),
        "every output must be reduce_sum": tl.relu(xs),
        "not row-chunked": tl.reduce_sum(tl.add(xs, c((64, 16), 3)), [0]),
    }
    for msg, out in bad.items():
        with pytest.raises(RuntimeError, match=msg):
            tl.Plan([out], pipeline_chunks=2)
    with pytest.raises(RuntimeError, match="streamed rank-2 batch input"):
        tl.Plan([tl.reduce_sum(tl.relu(c((8, 8))), [0])], pipeline_chunks=2)
    with pytest.raises(RuntimeError, match="chunks must be"):
        tl.Plan([tl.reduce_sum(tl.relu(xs), [0])], pipeline_chunks=65)


def test_dag_stress_workload_drops_dead_operations_and_fuses():
    """The DCE / fusion stress graph (bench.py's dag_stress at a small size):
    no unreachable operation reaches the tape, and fusion leaves fewer tape
    operations than live graph operations."""
    from tt_lazy_b200 import workloads

    outs, work = workloads.dag_stress(n=32, nodes=200)
    assert work["dead_ops"] == 80 and work["graph_nodes"] == 204
    t = tl.tape(outs)
    taped = set()
    for op in t:
        taped.add(op["node"])
        taped.update(op["outputs"])
    assert sum(op["fused_nodes"] for op in t) <= work["live_ops"]
    assert len(t) < work["live_ops"]
    # every taped node is an ancestor of an output: nothing from the dead part
    produced = set()
    for op in t:
        for i in op["inputs"]:
            assert i in produced or i not in taped
        produced.update(op["outputs"])
        produced.add(op["node"])


def test_gemm_path_names_are_checked():
    with pytest.raises(ValueError, match="auto, ffma, tf32 or tf32x3"):
        tl.set_gemm_path("fp64")
    for p in ("ffma", "tf32", "tf32x3", "auto"):
        tl.set_gemm_path(p)
