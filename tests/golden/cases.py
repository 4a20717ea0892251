"""Small graph cases shared by the golden-fixture generator and the tests.

Each case is (name, inputs, build).  ``build(g, t)`` creates the graph with a
builder ``g`` (methods: fused(a, b, steps), matmul(a, b), add(a, b), relu(x);
steps are ("add", node) / ("relu", None)) and ``t``, a dict of input nodes by
name; it returns the root.  Graphs are written in the form MiniXLA's
optimize() leaves them (OP_FUSED nodes), so the same build runs on the
reference's host API and on the ctypes mirror.

Sources of the cases (gouthamk16/miniXLA):
  tests.c:92-107   relu(AB + C)          expects {0, 28, 49, 0}
  tests.c:48-65    relu(AB + bias[N])    expects {0, 0, 19, 4}
  tests.c:191-220  diamond epilogue      expects {5, 4, 11, 10}
  gpu_test.c:83-126, 132-188, 201-249  diamond / two-layer / deep-chain fills
plus seeded cases at the benchmark shapes scaled down, ragged tile edges, the
modulo-operand rule of graph.c:100-105, and the 3-layer MLP DAG.
"""
from __future__ import annotations

import numpy as np

from minixla_b200 import datagen


def _u(shape, stream):
    return datagen.uniform(shape, stream)


def _n(shape, stream, mu=0.0, sigma=1.0):
    return datagen.normal(shape, stream, mu, sigma)


def _fill(n, f):
    return np.array([f(i) for i in range(n)], dtype=np.float32)


def case_tests_fused_exec():
    a = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    b = np.arange(1, 7, dtype=np.float32).reshape(3, 2)
    c = np.array([[-100, 0], [0, -100]], dtype=np.float32)
    return "tests_fused_exec", {"a": a, "b": b, "c": c}, \
        lambda g, t: g.fused(t["a"], t["b"], [("add", t["c"]), ("relu", None)])


def case_tests_bias():
    a = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    b = np.arange(1, 7, dtype=np.float32).reshape(3, 2)
    bias = np.array([-30, -60], dtype=np.float32)
    return "tests_bias", {"a": a, "b": b, "bias": bias}, \
        lambda g, t: g.fused(t["a"], t["b"], [("add", t["bias"]), ("relu", None)])


def case_tests_diamond():
    x = np.array([[1, 2], [3, 4]], dtype=np.float32)
    w1 = np.array([[1, 0], [0, 1]], dtype=np.float32)
    w2 = np.array([[0, 1], [1, 0]], dtype=np.float32)
    w3 = np.ones((2, 2), dtype=np.float32)

    def build(g, t):
        h1 = g.fused(t["x"], t["w1"], [("relu", None)])
        h2 = g.fused(t["x"], t["w2"], [("relu", None)])
        return g.fused(h1, t["w3"], [("add", h2)])

    return "tests_diamond", {"x": x, "w1": w1, "w2": w2, "w3": w3}, build


def case_gpu_two_layer():
    M, K1, N1, N2 = 4, 8, 16, 4
    x = _fill(M * K1, lambda i: (i % 5) * 0.1).reshape(M, K1)
    w1 = _fill(K1 * N1, lambda i: (i % 7) * 0.05 - 0.1).reshape(K1, N1)
    b1 = _fill(M * N1, lambda i: (i % 3) * 0.02).reshape(M, N1)
    w2 = _fill(N1 * N2, lambda i: (i % 11) * 0.03 - 0.15).reshape(N1, N2)
    b2 = _fill(M * N2, lambda i: (i % 4) * 0.01).reshape(M, N2)

    def build(g, t):
        hidden = g.fused(t["x"], t["w1"], [("add", t["b1"]), ("relu", None)])
        return g.fused(hidden, t["w2"], [("add", t["b2"])])

    return "gpu_two_layer", {"x": x, "w1": w1, "b1": b1, "w2": w2, "b2": b2}, build


def case_gpu_deep_chain(S=64, layers=8):
    x = _fill(S * S, lambda i: (i % 13) * 0.01 - 0.06).reshape(S, S)
    ws = {f"w{l}": _fill(S * S, lambda i, l=l: ((i + l) % 11) * 0.01 - 0.05).reshape(S, S) for l in range(layers)}

    def build(g, t):
        h = t["x"]
        for l in range(layers):
            h = g.fused(h, t[f"w{l}"], [("relu", None)])
        return h

    return "gpu_deep_chain", {"x": x, **ws}, build


def case_config1():
    A, B, C = _u((128, 128), 0), _u((128, 128), 1), _u((128, 128), 2)
    return "config1_128", {"A": A, "B": B, "C": C}, \
        lambda g, t: g.fused(t["A"], t["B"], [("add", t["C"]), ("relu", None)])


def case_ragged(M, N, K, tag):
    A, B, C = _u((M, K), 10), _u((K, N), 11), _u((M, N), 12)
    return f"ragged_{tag}", {"A": A, "B": B, "C": C}, \
        lambda g, t: g.fused(t["A"], t["B"], [("add", t["C"]), ("relu", None)])


def case_bias_chain():
    M, N, K = 130, 140, 70
    A, B = _u((M, K), 20), _u((K, N), 21)
    bias, C = _n((N,), 22, 0.0, 0.1), _n((M, N), 23)
    return "bias_chain", {"A": A, "B": B, "bias": bias, "C": C}, \
        lambda g, t: g.fused(t["A"], t["B"], [("add", t["bias"]), ("relu", None), ("add", t["C"]),
                                              ("relu", None), ("add", t["bias"])])


def case_mod_operand():
    M, N, K = 37, 29, 19
    A, B, op = _u((M, K), 30), _u((K, N), 31), _u((7,), 32)
    return "mod_operand", {"A": A, "B": B, "op": op}, \
        lambda g, t: g.fused(t["A"], t["B"], [("add", t["op"]), ("relu", None)])


def case_bare_and_standalone():
    M, N, K = 40, 36, 24
    A, B, C, bias = _u((M, K), 40), _u((K, N), 41), _u((M, N), 42), _u((N,), 43)

    def build(g, t):
        mm = g.matmul(t["A"], t["B"])           # bare matmul: never fused by optimize()
        s = g.add(mm, t["C"])                   # standalone add (same shape)
        s = g.add(s, t["bias"])                 # standalone add (bias row broadcast)
        return g.relu(s)                        # standalone relu

    return "bare_and_standalone", {"A": A, "B": B, "C": C, "bias": bias}, build


def case_mlp_small(M=64, D=32, H=64):
    X = _u((M, D), 50)
    W1 = _n((D, H), 51, 0.0, 1.0 / np.sqrt(D))
    W2 = _n((H, H), 52, 0.0, 1.0 / np.sqrt(H))
    W2p = _n((H, H), 53, 0.0, 1.0 / np.sqrt(H))
    W3 = _n((H, D), 54, 0.0, 1.0 / np.sqrt(H))
    b1, b2, b3 = _n((H,), 55, 0.0, 0.1), _n((H,), 56, 0.0, 0.1), _n((D,), 57, 0.0, 0.1)

    def build(g, t):
        # The structure optimize() gives the 3-layer MLP of the benchmark
        # configs: F1 = [ADD b1, RELU]; F2 = [ADD b2, RELU, ADD (h W2')] with
        # h W2' left as a bare matmul; F3 = [ADD b3].
        h = g.fused(t["X"], t["W1"], [("add", t["b1"]), ("relu", None)])
        hw = g.matmul(h, t["W2p"])
        y = g.fused(h, t["W2"], [("add", t["b2"]), ("relu", None), ("add", hw)])
        return g.fused(y, t["W3"], [("add", t["b3"])])

    return "mlp_small", {"X": X, "W1": W1, "W2": W2, "W2p": W2p, "W3": W3, "b1": b1, "b2": b2, "b3": b3}, build


def case_batched():
    """Rank-3 fused node: eval_fused runs batches (graph.c:80-113); ADD
    operands holding every batch, one M x N block, a [N] row, and an odd size
    read by the modulo rule over the flat batched index."""
    bt, M, N, K = 3, 37, 29, 21
    A, B = _u((bt, M, K), 90), _u((bt, K, N), 91)
    C, blk = _n((bt, M, N), 92), _u((M, N), 93)
    bias, odd = _n((N,), 94, 0.0, 0.5), _u((11,), 95)
    return "batched_rank3", {"A": A, "B": B, "C": C, "blk": blk, "bias": bias, "odd": odd}, \
        lambda g, t: g.fused(t["A"], t["B"], [("add", t["C"]), ("relu", None), ("add", t["blk"]),
                                              ("add", t["bias"]), ("add", t["odd"])])


def all_cases():
    return [
        case_tests_fused_exec(), case_tests_bias(), case_tests_diamond(),
        case_gpu_two_layer(), case_gpu_deep_chain(), case_config1(),
        case_ragged(1, 257, 129, "1x257x129"), case_ragged(129, 127, 33, "129x127x33"),
        case_ragged(257, 264, 129, "257x264x129"), case_ragged(7, 4097, 5, "7x4097x5"),
        case_bias_chain(), case_mod_operand(), case_bare_and_standalone(), case_mlp_small(),
        case_batched(),
    ]


# Longest chain of GEMMs from an input to the root.  The tolerances
# are per fused op; rounding error compounds through chained layers, so
# graph-level checks scale the tolerance by this depth.
DEPTH = {"tests_diamond": 2, "gpu_two_layer": 2, "gpu_deep_chain": 8, "mlp_small": 3}

# Known answers printed in the reference's own tests.
KNOWN_ANSWERS = {
    "tests_fused_exec": [0, 28, 49, 0],      # tests.c:102
    "tests_bias": [0, 0, 19, 4],             # tests.c:60
    "tests_diamond": [5, 4, 11, 10],         # tests.c:215
}
