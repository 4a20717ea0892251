"""CPU tests: the oracle is pinned to MiniXLA's own results before it is trusted.

* bit-exact against the golden fixture (outputs of the reference's execute());
* the known answers printed in the reference's tests.c;
* bit-exact against the reference's execute() on fresh seeded cases (where
  its host library was built here from the reference sources);
* the optimize() pass of the reference produces the fused structures the
  cases are written in.
"""
import hashlib

import numpy as np
import pytest

from oracle import bindings
from tests.golden.cases import KNOWN_ANSWERS, all_cases
from tests.graph_eval import oracle_eval

CASES = all_cases()


def _digest(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return hashlib.sha256(repr(a.shape).encode() + a.tobytes()).hexdigest()


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_inputs_match_fixture(case, golden):
    name, inputs, _ = case
    for k, v in inputs.items():
        assert str(golden[f"{name}:{k}:sha256"]) == _digest(v), f"{name}:{k} generator drifted"


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_oracle_bit_exact_vs_golden(case, golden):
    name, inputs, build = case
    got = oracle_eval(inputs, build)
    want = golden[f"{name}:__out__"]
    assert got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"{name}: oracle differs from execute()"


@pytest.mark.parametrize("name", sorted(KNOWN_ANSWERS))
def test_known_answers(name, golden):
    case = next(c for c in CASES if c[0] == name)
    got = oracle_eval(case[1], case[2])
    np.testing.assert_allclose(got.reshape(-1), KNOWN_ANSWERS[name], atol=1e-4)
    np.testing.assert_allclose(golden[f"{name}:__out__"].reshape(-1), KNOWN_ANSWERS[name], atol=1e-4)


def test_oracle_f64_close_to_f32():
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (33, 300)).astype(np.float32)
    B = rng.uniform(-1, 1, (300, 45)).astype(np.float32)
    C = rng.normal(size=(33, 45)).astype(np.float32)
    f32 = bindings.fused_oracle(A, B, [("add", C), ("relu",)])
    f64 = bindings.fused_oracle(A, B, [("add", C), ("relu",)], f64=True)
    exact = np.maximum(A.astype(np.float64) @ B.astype(np.float64) + C, 0)
    assert np.max(np.abs(f64 - exact)) < 1e-10
    assert np.max(np.abs(f32 - exact)) < 1e-4


def test_oracle_row_sample_matches_full():
    rng = np.random.default_rng(1)
    A = rng.uniform(-1, 1, (50, 20)).astype(np.float32)
    B = rng.uniform(-1, 1, (20, 30)).astype(np.float32)
    bias = rng.normal(size=(30,)).astype(np.float32)
    full = bindings.fused_oracle(A, B, [("add", bias), ("relu",)])
    rows = [0, 7, 49, 13]
    part = bindings.fused_oracle(A, B, [("add", bias), ("relu",)], rows=rows, threads=3)
    assert np.array_equal(part, full[rows])


def test_oracle_scale_step_matches_f64():
    # SCALE has no reference op: it is checked against float64 only.
    rng = np.random.default_rng(2)
    A = rng.uniform(-1, 1, (8, 16)).astype(np.float32)
    B = rng.uniform(-1, 1, (16, 8)).astype(np.float32)
    got = bindings.fused_oracle(A, B, [("scale", 0.5), ("relu",)])
    want = np.maximum(0.5 * (A.astype(np.float64) @ B.astype(np.float64)), 0)
    np.testing.assert_allclose(got, want, atol=1e-5)


def test_oracle_add_relu_elementwise():
    a = np.arange(12, dtype=np.float32).reshape(3, 4) - 6
    b = np.array([1, -2, 3, -4], dtype=np.float32)
    np.testing.assert_array_equal(bindings.add_oracle(a, b), a + b)
    np.testing.assert_array_equal(bindings.relu_oracle(a), np.where(a > 0, a, 0))


# ---------------------------------------------------------------- vs the reference itself

needs_ref = pytest.mark.skipif(not bindings.ref_available(), reason="reference host library not built here")


@needs_ref
@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 5, 7), (64, 48, 40), (129, 130, 67), (5, 300, 257)])
def test_oracle_bit_exact_vs_reference_execute(shape):
    from minixla_b200.abi import OP_ADD, OP_RELU

    M, N, K = shape
    rng = np.random.default_rng(M * 1000 + N)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    C = rng.normal(size=(M, N)).astype(np.float32)
    bias = rng.normal(size=(N,)).astype(np.float32)
    rg = bindings.RefGraph()
    try:
        root = rg.own(rg.fused(rg.input(A), rg.input(B),
                               [(OP_ADD, rg.input(C)), (OP_RELU, None), (OP_ADD, rg.input(bias))]))
        want = rg.execute(root)
    finally:
        rg.close()
    got = bindings.fused_oracle(A, B, [("add", C), ("relu",), ("add", bias)])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@needs_ref
def test_reference_optimize_yields_case_structure():
    """optimize() of the 3-layer MLP written with g_* gives F1/F2/F3 + one bare matmul."""
    from minixla_b200.abi import OP_ADD, OP_FUSED, OP_MATMUL, OP_RELU

    name, inputs, build = next(c for c in CASES if c[0] == "mlp_small")
    rg = bindings.RefGraph()
    L = rg.lib
    try:
        t = {k: rg.input(v) for k, v in inputs.items()}
        h = L.g_relu(L.g_add(L.g_matmul(t["X"], t["W1"]), t["b1"]))
        y = L.g_add(L.g_relu(L.g_add(L.g_matmul(h, t["W2"]), t["b2"])), L.g_matmul(h, t["W2p"]))
        out = L.g_add(L.g_matmul(y, t["W3"]), t["b3"])
        root = rg.own(rg.optimize(out))
        f3 = root.contents
        assert f3.op == OP_FUSED and f3.n_epilogue == 1 and f3.epilogue[0].op == OP_ADD
        f2 = f3.inputs[0].contents
        assert f2.op == OP_FUSED
        assert [f2.epilogue[i].op for i in range(f2.n_epilogue)] == [OP_ADD, OP_RELU, OP_ADD]
        assert f2.epilogue[2].operand.contents.op == OP_MATMUL
        f1 = f2.inputs[0].contents
        assert f1.op == OP_FUSED and [f1.epilogue[i].op for i in range(f1.n_epilogue)] == [OP_ADD, OP_RELU]
        got = rg.execute(root)
    finally:
        rg.close()
    want = oracle_eval(inputs, build)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
