"""Graph builders for the smaller benchmark workloads, through the public
front end (the same calls a user makes):

- ``readme_chain``: the README chain, x ~ U(-1,1) (seed 0), y = relu(x),
  z = add(y, y), w = multiply(z, z), s = reduce_sum(w); outputs w and s
  (reference README and tests/cpp/integration/test_end_to_end.cpp).
- ``small_mlp``: X[256,512] ~ N(0,1), W1[512,1024], W2[1024,512] ~
  N(0,1/fan_in), b1, b2 ~ U(-0.1,0.1) (seed 1); relu(X W1 + b1) W2 + b2,
  then reduce_mean over rows (exercises MLP fusion and dead-code elimination).
- ``dag_stress``: a random DAG of ``nodes`` operations (seed 4) over
  [n, n] tensors mixing matmul / relu / sigmoid / add / multiply, with
  reduce_sum at the sinks and ``dead_frac`` of the operations unreachable
  from the outputs (tape build, dead-code elimination and fusion under load);
  ``dag_stress_program`` draws its data and topology and ``dag_build``
  creates the graph nodes, so the two can be timed apart and the program
  replayed on the oracle.

Inputs are seeded synthetic data with the workloads' shapes and
distributions. Each builder returns the lazy outputs plus a description of
the algorithmic work (bytes moved, flops) that a throughput figure divides;
for the DAG, ``bytes_unfused`` counts every operation reading its inputs and
writing its result once, as an unfused evaluation would.
"""
from __future__ import annotations

import numpy as np

import tt_lazy_b200 as tl


def readme_chain(n: int = 1000, m: int | None = None, seed: int = 0):
    """(w, s, work): the README chain over an n x m input (m defaults to n)."""
    m = n if m is None else m
    x = np.random.default_rng(seed).uniform(-1, 1, (n, m)).astype(np.float32)
    y = tl.relu(tl.constant(x))
    z = tl.add(y, y)
    w = tl.multiply(z, z)
    s = tl.reduce_sum(w)
    work = {"bytes": 2 * 4 * n * m + 4, "inputs": {"x": x}}
    return w, s, work


def small_mlp(seed: int = 1, batch: int = 256, d_in: int = 512, d_hidden: int = 1024, d_out: int = 512):
    """(m, work): reduce_mean over rows of relu(X W1 + b1) W2 + b2."""
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((batch, d_in)).astype(np.float32)
    W1 = (rng.standard_normal((d_in, d_hidden)) / np.sqrt(d_in)).astype(np.float32)
    W2 = (rng.standard_normal((d_hidden, d_out)) / np.sqrt(d_hidden)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, (1, d_hidden)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, (1, d_out)).astype(np.float32)
    h = tl.relu(tl.add(tl.matmul(tl.constant(X), tl.constant(W1)), tl.constant(b1)))
    y = tl.add(tl.matmul(h, tl.constant(W2)), tl.constant(b2))
    m = tl.reduce_mean(y, [0])
    work = {"flops": 2 * batch * d_in * d_hidden + 2 * batch * d_hidden * d_out,
            "inputs": {"X": X, "W1": W1, "b1": b1, "W2": W2, "b2": b2}}
    return m, work


def dag_stress_program(n: int = 4096, nodes: int = 200, seed: int = 4, dead_frac: float = 0.4, sinks: int = 4):
    """(inputs, program, work): the data and topology of the DCE / fusion
    stress graph, before any graph node exists.

    inputs: x0 [n, n] ~ U(-1, 1), two weights N(0, 1/n), two gates U(-1, 1).
    program: one (kind, a, b) per operation, operands numbered as values:
    0 = x0, 1 + i = operation i; b names a weight (matmul), a second value
    (add) or a gate / earlier sigmoid (multiply: "g0", "g1" or a value).
    The live part is a chain in which operation i always reads operation
    i - 1 (so every live operation reaches the last one) plus a second,
    random earlier operand for the binary ops; the dead part reads live or
    dead operations but feeds nothing. reduce_sum(dim 1) is taken at the last
    `sinks` live operations. Magnitudes stay bounded: matmul's right operand
    is a constant N(0, 1/n) matrix, multiply's second operand a constant in
    [-1, 1] or a sigmoid output, so only add grows values (by at most 2x).
    Every operation is row-local (matmul has a constant on the right), so
    row r of any value depends only on row r of x0 and of the gates."""
    rng = np.random.default_rng(seed)
    n_dead = int(round(nodes * dead_frac))
    n_live = nodes - n_dead
    inputs = {"x0": rng.uniform(-1, 1, (n, n)).astype(np.float32)}
    for i in range(2):
        inputs[f"w{i}"] = (rng.standard_normal((n, n)) / np.sqrt(n)).astype(np.float32)
    for i in range(2):
        inputs[f"g{i}"] = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    kinds = ["matmul", "relu", "sigmoid", "add", "multiply"]
    counts = dict.fromkeys(kinds, 0)
    program: list[tuple] = []
    sig_vals: list[int] = []

    def op(kind, prev, pool):
        if kind == "matmul":
            return (kind, prev, f"w{int(rng.integers(0, 2))}")
        if kind in ("relu", "sigmoid"):
            return (kind, prev, None)
        if kind == "add":
            return (kind, prev, pool[int(rng.integers(0, len(pool)))])
        bounded = ["g0", "g1"] + [v for v in sig_vals if v < len(pool)]
        return (kind, prev, bounded[int(rng.integers(0, len(bounded)))])

    live = [0]
    for _ in range(n_live):
        kind = kinds[int(rng.integers(0, len(kinds)))]
        counts[kind] += 1
        program.append(op(kind, live[-1], live))
        live.append(len(program))
        if kind == "sigmoid":
            sig_vals.append(len(live) - 1)
    dead: list[int] = []
    for _ in range(n_dead):
        kind = kinds[int(rng.integers(0, len(kinds)))]
        src = live + dead
        program.append(op(kind, src[int(rng.integers(0, len(src)))], src))
        dead.append(len(program))
    sink_vals = live[-sinks:]
    elem = 4 * n * n
    bytes_live = (counts["relu"] + counts["sigmoid"]) * 2 * elem + (counts["add"] + counts["multiply"]) * 3 * elem
    bytes_live += counts["matmul"] * 3 * elem + sinks * (elem + 4 * n)
    work = {"flops": counts["matmul"] * 2 * n ** 3, "bytes_unfused": bytes_live, "live_ops": n_live + sinks,
            "dead_ops": n_dead, "graph_nodes": nodes + sinks, "counts": counts, "sinks": sink_vals}
    return inputs, program, work


def dag_build(inputs: dict, program: list, sinks: list):
    """The lazy graph of a stress program: constants, one front-end call per
    operation, reduce_sum(dim 1) at the sink values. Returns the outputs."""
    const = {k: tl.constant(v) for k, v in inputs.items()}
    vals = [const["x0"]]
    for kind, a, b in program:
        if kind == "matmul":
            vals.append(tl.matmul(vals[a], const[b]))
        elif kind == "relu":
            vals.append(tl.relu(vals[a]))
        elif kind == "sigmoid":
            vals.append(tl.sigmoid(vals[a]))
        elif kind == "add":
            vals.append(tl.add(vals[a], vals[b]))
        else:
            vals.append(tl.multiply(vals[a], const[b] if isinstance(b, str) else vals[b]))
    return [tl.reduce_sum(vals[s], [1]) for s in sinks]


def dag_stress(n: int = 4096, nodes: int = 200, seed: int = 4, dead_frac: float = 0.4, sinks: int = 4):
    """(outputs, work): the stress graph built through the front end."""
    inputs, program, work = dag_stress_program(n, nodes, seed, dead_frac, sinks)
    return dag_build(inputs, program, work["sinks"]), work
