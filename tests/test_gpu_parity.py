"""GPU parity tests: the sm_100a path against the oracle, through the C ABI.

Tolerances (the accuracy targets of the fused path):
  3xTF32 mode: relative Frobenius error <= 1e-5 against MiniXLA's fp32 execute();
  TF32 mode:   relative Frobenius error <= 2e-3;
  both:        no NaN, and no sign flip after relu beyond what the tolerance
               allows (an output may only change sign / zero-ness where the
               oracle value is within the error band of zero).
Small graphs with exactly representable values must match bit for bit.
"""
import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from minixla_b200 import datagen
from minixla_b200 import lib as mlib
from minixla_b200.abi import OP_ADD, OP_MUL, OP_RELU, HostGraph, free_host_tensor, tensor_to_numpy
from oracle import bindings
from tests.golden.cases import DEPTH, KNOWN_ANSWERS, all_cases
from tests.graph_eval import HostBuilder, host_graph, oracle_eval, rel_frobenius

pytestmark = pytest.mark.gpu

TF32, X3 = mlib.GPU_PRECISION_TF32, mlib.GPU_PRECISION_3XTF32
TOL = {TF32: 2e-3, X3: 1e-5}
CASES = all_cases()
ROOT = Path(__file__).resolve().parents[1]


def run_execute(lib, ctx, root, precision):
    assert lib.gpu_ctx_set_precision(ctx, precision) == 0
    t = lib.gpu_execute(root, ctx)
    assert t, f"gpu_execute failed: {mlib.last_error()}"
    try:
        return tensor_to_numpy(t)
    finally:
        free_host_tensor(t)


def check(got, want, precision, what="", band=None, depth=1):
    assert got.shape == want.shape, what
    assert not np.isnan(got).any(), f"{what}: NaN in GPU output"
    tol = depth * TOL[precision]
    err = rel_frobenius(got, want)
    assert err <= tol, f"{what}: relative Frobenius {err:.3g} > {tol:g}"
    # Zero / sign agreement after relu: only where the oracle is clearly away from 0.
    band = band if band is not None else 50 * tol * (np.abs(want).max() + 1e-30)
    clear = np.abs(want) > band
    assert np.array_equal(np.sign(got[clear]), np.sign(want[clear])), f"{what}: sign flips"
    return err


# ---------------------------------------------------------------- golden cases


@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_golden_case(lib, gpu_ctx, golden, case, precision):
    name, inputs, build = case
    hg, root = host_graph(inputs, build)
    got = run_execute(lib, gpu_ctx, root, precision)
    want = golden[f"{name}:__out__"]
    check(got, want, precision, name, depth=DEPTH.get(name, 1))
    if name in KNOWN_ANSWERS:  # small integers: exact in every mode
        assert np.array_equal(got.reshape(-1), np.array(KNOWN_ANSWERS[name], dtype=np.float32))


def test_gpu_execute_leaves_graph_untouched(lib, gpu_ctx):
    name, inputs, build = next(c for c in CASES if c[0] == "mlp_small")
    hg, root = host_graph(inputs, build)
    before = bytes(C.string_at(C.addressof(root.contents), C.sizeof(root.contents)))
    run_execute(lib, gpu_ctx, root, X3)
    assert bytes(C.string_at(C.addressof(root.contents), C.sizeof(root.contents))) == before
    assert not root.contents.output


# ---------------------------------------------------------------- reference host API + optimize()

needs_ref = pytest.mark.skipif(not bindings.ref_available(), reason="reference host library not shipped")


@needs_ref
@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
def test_reference_graph_through_optimize(lib, gpu_ctx, precision):
    """A graph built and optimized by MiniXLA's own code runs unchanged on this backend."""
    name, inputs, build = next(c for c in CASES if c[0] == "mlp_small")
    rg = bindings.RefGraph()
    L = rg.lib
    try:
        t = {k: rg.input(v) for k, v in inputs.items()}
        h = L.g_relu(L.g_add(L.g_matmul(t["X"], t["W1"]), t["b1"]))
        y = L.g_add(L.g_relu(L.g_add(L.g_matmul(h, t["W2"]), t["b2"])), L.g_matmul(h, t["W2p"]))
        root = rg.own(rg.optimize(L.g_add(L.g_matmul(y, t["W3"]), t["b3"])))
        got = run_execute(lib, gpu_ctx, root, precision)  # before execute() memoizes anything
        want = rg.execute(root)
    finally:
        rg.close()
    check(got, want, precision, "mlp via optimize()", depth=DEPTH["mlp_small"])


# ---------------------------------------------------------------- gpu_test.c mirrors


def test_single_fused_via_gpu_run_fused(lib):
    """gpu_test.c:21-41: 2x3 . 3x2 + C, relu through gpu_run_fused, tol 1e-4."""
    name, inputs, build = next(c for c in CASES if c[0] == "tests_fused_exec")
    hg, root = host_graph(inputs, build)
    t = lib.gpu_run_fused(root, b"ignored ptx")
    assert t, mlib.last_error()
    got = tensor_to_numpy(t)
    free_host_tensor(t)
    np.testing.assert_allclose(got.reshape(-1), KNOWN_ANSWERS[name], atol=1e-4)


def test_broadcast_bias_now_supported(lib, gpu_ctx):
    """gpu_test.c:48-73 asserted that a [N] bias was refused on the GPU; this
    backend runs it (eval_fused's broadcast rule, graph.c:100-105) and must
    match execute(): {0, 0, 19, 4} (tests.c:48-65)."""
    name, inputs, build = next(c for c in CASES if c[0] == "tests_bias")
    hg, root = host_graph(inputs, build)
    np.testing.assert_array_equal(run_execute(lib, gpu_ctx, root, X3).reshape(-1), [0, 0, 19, 4])
    t = lib.gpu_run_fused(root, None)
    assert t
    np.testing.assert_array_equal(tensor_to_numpy(t).reshape(-1), [0, 0, 19, 4])
    free_host_tensor(t)
    t = lib.gpu_run_tensorcore(root, gpu_ctx)
    assert t
    np.testing.assert_array_equal(tensor_to_numpy(t).reshape(-1), [0, 0, 19, 4])
    free_host_tensor(t)


@pytest.mark.parametrize("name,tol", [("tests_diamond", 1e-3), ("gpu_two_layer", 1e-3), ("gpu_deep_chain", 5e-2)])
def test_gpu_test_graphs_default_mode(lib, gpu_ctx, golden, name, tol):
    """gpu_test.c:83-126, 132-188, 201-249 with their absolute tolerances, default precision."""
    case = next(c for c in CASES if c[0] == name)
    hg, root = host_graph(case[1], case[2])
    lib.gpu_ctx_set_precision(gpu_ctx, X3)
    t = lib.gpu_execute(root, gpu_ctx)
    assert t
    got = tensor_to_numpy(t)
    free_host_tensor(t)
    assert np.max(np.abs(got - golden[f"{name}:__out__"])) <= tol


def test_deep_chain_returns_memory(lib):
    """gpu_test.c:230-241: device memory back to baseline (within 16 MiB) once
    the context that ran the graph is destroyed."""
    import torch

    name, inputs, build = next(c for c in CASES if c[0] == "gpu_deep_chain")
    hg, root = host_graph(inputs, build)
    torch.cuda.init()
    free0, _ = torch.cuda.mem_get_info(0)
    ctx = lib.gpu_ctx_create()
    t = lib.gpu_execute(root, ctx)
    assert t
    free_host_tensor(t)
    lib.gpu_ctx_destroy(ctx)
    free1, _ = torch.cuda.mem_get_info(0)
    assert free1 >= free0 - 16 * 1024 * 1024


def test_module_cache_same_graph_twice(lib, gpu_ctx, golden):
    """gpu_test.c:254-281: the same graph twice on one context gives the same answer."""
    case = next(c for c in CASES if c[0] == "config1_128")
    hg, root = host_graph(case[1], case[2])
    r1 = run_execute(lib, gpu_ctx, root, X3)
    r2 = run_execute(lib, gpu_ctx, root, X3)
    assert np.array_equal(r1, r2)
    check(r1, golden["config1_128:__out__"], X3)


def test_large_relu_matmul_512(lib, gpu_ctx):
    """gpu_test.c:286-335: relu(512^2 matmul), tol 1e-2, integer-pattern fills."""
    S = 512
    a = (((np.arange(S * S) % 17) * 0.01) - 0.08).astype(np.float32).reshape(S, S)
    b = (((np.arange(S * S) % 13) * 0.01) - 0.06).astype(np.float32).reshape(S, S)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(a), hg.input_node(b), [(OP_RELU, None)])
    want = bindings.fused_oracle(a, b, [("relu",)])
    for p in (X3, TF32):
        got = run_execute(lib, gpu_ctx, root, p)
        assert np.max(np.abs(got - want)) <= 1e-2


def _tc_values(shape, stream):
    # gpu_test.c:359-365 fills with (rand() % 2000 - 1000) / 100: multiples of 0.01 in [-10, 10).
    u = datagen.raw_bits(int(np.prod(shape)), stream) % np.uint64(2000)
    return ((u.astype(np.int64) - 1000) / 100.0).astype(np.float32).reshape(shape)


@pytest.mark.parametrize("mkn", [(16, 8, 8), (17, 8, 8), (16, 8, 9), (16, 5, 8), (100, 100, 100), (1024, 1024, 1024),
                                 (2048, 2048, 2049)])
def test_tensorcore_correctness(lib, gpu_ctx, mkn):
    """gpu_test.c:393-403 through gpu_run_tensorcore, with its tolerance
    atol = 0.05 sqrt(K), rtol = 0.02 (gpu_test.c:349-357)."""
    M, K, N = mkn
    a, b = _tc_values((M, K), 60), _tc_values((K, N), 61)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(a), hg.input_node(b), [])
    t = lib.gpu_run_tensorcore(root, gpu_ctx)
    assert t, mlib.last_error()
    got = tensor_to_numpy(t)
    free_host_tensor(t)
    want = bindings.fused_oracle(a, b, [])
    assert np.all(np.abs(got - want) <= 0.05 * np.sqrt(K) + 0.02 * np.abs(want))


def test_tensorcore_epilogue(lib, gpu_ctx):
    """gpu_test.c:407-430: 100^3 with ADD + RELU through the TF32 path."""
    a, b, c = _tc_values((100, 100), 62), _tc_values((100, 100), 63), _tc_values((100, 100), 64)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(a), hg.input_node(b), [(OP_ADD, hg.input_node(c)), (OP_RELU, None)])
    t = lib.gpu_run_tensorcore(root, gpu_ctx)
    assert t
    got = tensor_to_numpy(t)
    free_host_tensor(t)
    want = bindings.fused_oracle(a, b, [("add", c), ("relu",)])
    assert np.all(np.abs(got - want) <= 0.05 * np.sqrt(100) + 0.02 * np.abs(want))


def test_kernel_timers(lib, gpu_ctx):
    """gpu_time_kernel_ms / _tc_ms return a positive minimum; -1.0 for a non-fused root."""
    case = next(c for c in CASES if c[0] == "config1_128")
    hg, root = host_graph(case[1], case[2])
    assert lib.gpu_time_kernel_ms(root, gpu_ctx, 3, 5) > 0
    assert lib.gpu_time_kernel_tc_ms(root, gpu_ctx, 3, 5) > 0
    mm = hg.g_matmul(hg.input_node(case[1]["A"]), hg.input_node(case[1]["B"]))
    assert lib.gpu_time_kernel_ms(mm, gpu_ctx, 1, 1) == -1.0


# ---------------------------------------------------------------- benchmark workloads


def _relu_abc(M, N, K, c_normal):
    A = datagen.uniform((M, K), 0)
    B = datagen.uniform((K, N), 1)
    C = datagen.normal((M, N), 2) if c_normal else datagen.uniform((M, N), 2)
    return A, B, C


def _sample_rows(M, n=512, seed=0):
    rng = np.random.default_rng(seed)
    edge = {0, M - 1}
    for t in range(128, M, 128):
        edge |= {t - 1, t}
    rows = sorted(edge | set(rng.integers(0, M, size=n).tolist()))
    return np.array([r for r in rows if 0 <= r < M], dtype=np.int64)


@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
@pytest.mark.parametrize("S", [512, 1024, 2048, 4096, 8192])
def test_config2_square_sweep(lib, gpu_ctx, S, precision, host_threads):
    """Config 2 against the oracle: every output up to 4096^3, and at 8192^3
    every 128-row tile edge plus 1024 random rows (about 1150 rows)."""
    A, B, C = _relu_abc(S, S, S, c_normal=True)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(C)), (OP_RELU, None)])
    got = run_execute(lib, gpu_ctx, root, precision)
    rows = None if S <= 4096 else _sample_rows(S, 1024)
    want = bindings.fused_oracle(A, B, [("add", C), ("relu",)], rows=rows, threads=host_threads)
    check(got if rows is None else got[rows], want, precision, f"{S}^3")


@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
def test_oracle_noise_at_8192(lib, gpu_ctx, precision, host_threads):
    """At K = 8192 the fp32 oracle's own k-ordered sum carries error of the
    order of the 3xTF32 budget, so the result is also compared with the
    float64 restatement of the same loop on the sampled rows: GPU vs fp32
    oracle, GPU vs float64 and fp32 oracle vs float64 are all reported, and
    the GPU must meet the tolerance against both references."""
    S = 8192
    A, B, C = _relu_abc(S, S, S, c_normal=True)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(C)), (OP_RELU, None)])
    got = run_execute(lib, gpu_ctx, root, precision)
    rows = _sample_rows(S, 256, seed=3)
    steps = [("add", C), ("relu",)]
    f32 = bindings.fused_oracle(A, B, steps, rows=rows, threads=host_threads)
    f64 = bindings.fused_oracle(A, B, steps, rows=rows, f64=True, threads=host_threads)
    e_gpu_f32 = rel_frobenius(got[rows], f32)
    e_gpu_f64 = rel_frobenius(got[rows], f64)
    e_f32_f64 = rel_frobenius(f32, f64)
    print(f"\n8192^3 {'tf32' if precision == TF32 else '3xtf32'}: gpu vs fp32 oracle {e_gpu_f32:.3g}, "
          f"gpu vs float64 {e_gpu_f64:.3g}, fp32 oracle vs float64 {e_f32_f64:.3g}")
    assert e_gpu_f32 <= TOL[precision] and e_gpu_f64 <= TOL[precision]
    assert e_f32_f64 < 1e-5


@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
@pytest.mark.parametrize("mnk", [(1000, 1000, 1000), (257, 4097, 129), (8191, 127, 3000), (1, 4096, 4096)])
def test_config3_ragged(lib, gpu_ctx, mnk, precision, host_threads):
    M, N, K = mnk
    A, B, C = _relu_abc(M, N, K, c_normal=False)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(C)), (OP_RELU, None)])
    got = run_execute(lib, gpu_ctx, root, precision)
    want = bindings.fused_oracle(A, B, [("add", C), ("relu",)], threads=host_threads)
    check(got, want, precision, f"{mnk}")


def _mlp_inputs(M=4096, D=1024, H=4096):
    return {
        "X": datagen.uniform((M, D), 70),
        "W1": datagen.normal((D, H), 71, 0.0, 1.0 / np.sqrt(D)),
        "W2": datagen.normal((H, H), 72, 0.0, 1.0 / np.sqrt(H)),
        "W2p": datagen.normal((H, H), 73, 0.0, 1.0 / np.sqrt(H)),
        "W3": datagen.normal((H, D), 74, 0.0, 1.0 / np.sqrt(H)),
        "b1": datagen.normal((H,), 75, 0.0, 0.1),
        "b2": datagen.normal((H,), 76, 0.0, 0.1),
        "b3": datagen.normal((D,), 77, 0.0, 0.1),
    }


@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
def test_three_layer_mlp_dag(lib, gpu_ctx, precision, host_threads):
    """3-layer MLP with a shared node (h feeds W2 and W2'), at full size.
    Rows are independent through every layer, so the oracle evaluates a row sample of X."""
    inp = _mlp_inputs()
    build = next(c for c in CASES if c[0] == "mlp_small")[2]
    hg, root = host_graph(inp, build)
    got = run_execute(lib, gpu_ctx, root, precision)
    rows = _sample_rows(4096, 128)
    sub = dict(inp, X=inp["X"][rows])
    want = oracle_eval(sub, build)
    check(got[rows], want, precision, "mlp")


@pytest.mark.parametrize("precision", [X3, TF32], ids=["3xtf32", "tf32"])
def test_full_size_checksums(lib, gpu_ctx, precision):
    """Size-independent check over every tile at the largest single-GPU shape:
    for out = A.B + C, column sums equal (1^T A) B + 1^T C and row sums equal
    A (B 1) + C 1 (float64 on the host)."""
    M, N, K = 8192, 8192, 8192
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(C))])
    got = run_execute(lib, gpu_ctx, root, precision).astype(np.float64)
    A64, B64, C64 = A.astype(np.float64), B.astype(np.float64), C.astype(np.float64)
    col_want = A64.sum(0) @ B64 + C64.sum(0)
    row_want = A64 @ B64.sum(1) + C64.sum(1)
    tol = 5 * TOL[precision]
    assert rel_frobenius(got.sum(0), col_want) < tol
    assert rel_frobenius(got.sum(1), row_want) < tol


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("variant", ["pair", "pair512", "single", "single64", "single32", "ksplit3"])
@pytest.mark.parametrize("mnk", [(256, 256, 32), (300, 520, 100), (1000, 1000, 1000), (257, 4097, 129),
                                 (8191, 127, 3000), (2048, 2048, 2048), (4096, 300, 1024), (640, 384, 4100)])
def test_kernel_variants(lib, gpu_ctx, mnk, variant, precision, monkeypatch, host_threads):
    """Every kernel of each mode (CTA pair with 256- and, in TF32, 512-wide
    tiles; single CTA with 128/256-, 64- and 32-wide tiles; the single-CTA
    kernel with K split three ways) on tile-edge shapes, with a
    full-matrix add, a bias row and relu in the epilogue.  K = 4100 ends on a
    partial k-block and a partial 3xTF32 segment."""
    if variant == "pair512" and precision == X3:
        pytest.skip("TF32-only kernel form")
    if variant == "ksplit3":
        monkeypatch.setenv("MINIXLA_KSPLIT", "3")
        variant = "single"
    if variant.startswith("single") and variant != "single":
        monkeypatch.setenv("MINIXLA_SINGLE_BN", variant[len("single"):])
        variant = "single"
    monkeypatch.setenv("MINIXLA_GEMM_VARIANT", variant)
    M, N, K = mnk
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    bias = datagen.normal((N,), 5, 0.0, 0.5)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_RELU, None), (OP_ADD, hg.input_node(bias))])
    got = run_execute(lib, gpu_ctx, root, precision)
    rows = None if M * N * K <= 2048 ** 3 else _sample_rows(M, 256)
    want = bindings.fused_oracle(A, B, [("add", C), ("relu",), ("add", bias)], rows=rows, threads=host_threads)
    check(got if rows is None else got[rows], want, precision, f"{variant} {mnk}")


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("mnk", [(8191, 127, 3000), (2047, 250, 6200), (2048, 256, 8192), (1024, 1024, 8192),
                                 (760, 890, 4100)])
def test_k_split(lib, gpu_ctx, mnk, precision, monkeypatch, host_threads):
    """Shapes whose 128 x 128 tiles fill under half the SMs with a long
    K (>= 64 k-blocks) run the single-CTA kernel with K split across CTAs
    (here two, three and four ways; (2047, 250, 6200) and (760, 890, 4100)
    end on a partial row tile, column tile and k-block): the result matches
    the oracle, repeats bit for bit (the slices are summed in slice order
    whichever CTA finishes last), equals the row-streamed executor's bit for
    bit (the split follows the node's full row count) and the separate reduce
    kernel's, and stays within tolerance of the unsplit kernel."""
    M, N, K = mnk
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    bias = datagen.normal((N,), 5, 0.0, 0.5)
    odd = datagen.uniform((13,), 6)  # read by eval_fused's modulo rule
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_ADD, hg.input_node(odd)), (OP_RELU, None),
                          (OP_ADD, hg.input_node(bias))])
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "1")
    got = run_execute(lib, gpu_ctx, root, precision)
    assert np.array_equal(got, run_execute(lib, gpu_ctx, root, precision)), "K-split result not repeatable"
    rows = _sample_rows(M, 256)
    want = bindings.fused_oracle(A, B, [("add", C), ("add", odd), ("relu",), ("add", bias)], rows=rows,
                                 threads=host_threads)
    check(got[rows], want, precision, f"k-split {mnk}")
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "8")
    assert np.array_equal(got, run_execute(lib, gpu_ctx, root, precision)), "row-streamed K split differs"
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "1")
    # The slices summed inside the GEMM's clusters (default) and by the
    # separate reduce kernel over workspace: the same additions, same bits.
    monkeypatch.setenv("MINIXLA_KSPLIT_REDUCE", "kernel")
    assert np.array_equal(got, run_execute(lib, gpu_ctx, root, precision)), "reduce kernel differs from cluster sum"
    monkeypatch.delenv("MINIXLA_KSPLIT_REDUCE")
    monkeypatch.setenv("MINIXLA_KSPLIT", "0")
    unsplit = run_execute(lib, gpu_ctx, root, precision)
    check(got, unsplit, precision, f"k-split vs unsplit {mnk}")
    assert not np.array_equal(got, unsplit), "same bits as the unsplit kernel: K was not split"


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
def test_row_streamed_executor_matches_one_stream(lib, gpu_ctx, precision, monkeypatch):
    """The row-streamed executor (uploads, kernels and downloads pipelined by
    row chunks over three streams) gives bit-identical results to the
    one-stream executor: every output element runs through the same kernel
    and k order either way.  Covers a FULL operand produced by another node
    (bare matmul -> ADD) and a standalone add + relu."""
    M, N, K = 1024, 768, 512
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    W = datagen.normal((N, N), 6, 0.0, 1.0 / np.sqrt(N))
    bias = datagen.normal((N,), 7, 0.0, 0.1)
    hg = HostGraph()
    a, b, c = hg.input_node(A), hg.input_node(B), hg.input_node(C)
    h = hg.fused_node(a, b, [(OP_ADD, c), (OP_RELU, None)])
    hw = hg.g_matmul(h, hg.input_node(W))
    y = hg.fused_node(h, hg.input_node(W), [(OP_ADD, hg.input_node(bias)), (OP_ADD, hw)])
    root = hg.g_relu(hg.g_add(y, hg.input_node(bias)))
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "1")
    one = run_execute(lib, gpu_ctx, root, precision)
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "8")
    streamed = run_execute(lib, gpu_ctx, root, precision)
    assert np.array_equal(one, streamed)
    # and into a caller buffer
    out = np.zeros((M, N), np.float32)
    assert lib.gpu_execute_into(root, gpu_ctx, hg.tensor(out)) == 0
    assert np.array_equal(out, streamed)


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("M", [1, 3, 8, 16])
@pytest.mark.parametrize("form,NK", [("cluster", (1000, 777)), ("split", (1000, 777)), ("cluster", (2501, 1500)),
                                     (None, (300, 20000))], ids=["cluster", "split", "cluster_wide", "long_k"])
def test_skinny_rows_path(lib, gpu_ctx, M, form, NK, precision, monkeypatch, host_threads):
    """Few output rows run on the split-K CUDA-core path (fp32): every
    epilogue kind, ragged N, against the oracle at the 3xTF32 tolerance.
    Both forms -- one kernel reducing over a cluster's shared memory, and
    partial sums + reduce kernel (MINIXLA_SKINNY_FORM=split) -- and K = 20000,
    whose slices of A do not fit in shared memory (two kernels by itself).
    TF32 mode sends 9 to 16 rows to the tensor-core kernel by default; the
    limit is raised here to cover the skinny kernels' 16-row forms."""
    monkeypatch.setenv("MINIXLA_SKINNY_MAX_ROWS", "16")
    if form:
        monkeypatch.setenv("MINIXLA_SKINNY_FORM", form)
    N, K = NK
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    bias = datagen.normal((N,), 8, 0.0, 0.5)
    odd = datagen.uniform((13,), 9)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_ADD, hg.input_node(odd)), (OP_RELU, None),
                          (OP_ADD, hg.input_node(bias))])
    got = run_execute(lib, gpu_ctx, root, precision)
    want = bindings.fused_oracle(A, B, [("add", C), ("add", odd), ("relu",), ("add", bias)], threads=host_threads)
    check(got, want, X3, f"skinny M={M}")


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("bmnk", [(16, 250, 130, 300), (5, 384, 520, 1000), (64, 128, 128, 128),
                                  (3, 1100, 1030, 1056)])
def test_batched_one_launch(lib, gpu_ctx, bmnk, precision, monkeypatch):
    """A rank-3 fused node whose products are small runs all of them in one
    launch (3-D tensor maps: a partial row tile or k-block of one product
    reads zeros, not the next product): ADD operands holding every product,
    one shared M x N block, a [N] row and an odd size read by the modulo rule
    over the flat batched index (graph.c:100-105), ragged M, N and K, on
    128- and (N >= 512, TF32) 256-wide tiles and, for 3 x (1100, 1030, 1056),
    the 256 x 256 tiles of the CTA-pair kernels of both modes.  The
    result matches the oracle and the one-launch-per-product loop
    (MINIXLA_BATCH_LAUNCH=0), and in TF32 mode the whole batch is one kernel
    launch."""
    from tests.graph_eval import host_graph, oracle_eval

    bt, M, N, K = bmnk
    if bmnk == (3, 1100, 1030, 1056):
        # This case is meant for the CTA-pair kernels: it reaches them only
        # when its 75 pair tiles give every CTA pair of this GPU one.
        import torch

        sms = torch.cuda.get_device_properties(lib.gpu_ctx_device(gpu_ctx)).multi_processor_count
        plan = mlib.gemm_plan(M, N, K, precision, sms, batch=bt)
        if plan.kernel != mlib.MXB_KERNEL_CTA_PAIR or plan.products != bt:
            pytest.skip(f"{sms} SMs: the batch does not run on the CTA-pair kernels in one launch")
    g = np.random.default_rng(bt * 1000 + M)
    inputs = {"A": g.uniform(-1, 1, (bt, M, K)).astype(np.float32),
              "B": g.uniform(-1, 1, (bt, K, N)).astype(np.float32),
              "C": g.normal(0, 1, (bt, M, N)).astype(np.float32),
              "blk": g.uniform(-1, 1, (M, N)).astype(np.float32),
              "bias": g.normal(0, 0.5, (N,)).astype(np.float32),
              "odd": g.uniform(-1, 1, (11,)).astype(np.float32)}

    def build(b, t):
        return b.fused(t["A"], t["B"], [("add", t["C"]), ("relu", None), ("add", t["blk"]), ("add", t["bias"]),
                                        ("add", t["odd"])])

    hg, root = host_graph(inputs, build)
    want = oracle_eval(inputs, build)
    n0 = lib.mxb_launch_count()
    got = run_execute(lib, gpu_ctx, root, precision)
    launches = lib.mxb_launch_count() - n0
    check(got, want, precision, f"batched {bmnk}")
    if precision == TF32:
        assert launches == 1, f"{launches} launches for {bt} products"
    monkeypatch.setenv("MINIXLA_BATCH_LAUNCH", "0")
    n0 = lib.mxb_launch_count()
    looped = run_execute(lib, gpu_ctx, root, precision)
    if precision == TF32:
        assert lib.mxb_launch_count() - n0 == bt
    check(got, looped, precision, f"batched {bmnk} one launch vs loop")


@pytest.mark.parametrize("M", [9, 16])
@pytest.mark.parametrize("NK", [(1000, 777), (2501, 8000)], ids=["short_k", "k_split"])
def test_few_rows_tensor_path(lib, gpu_ctx, M, NK, host_threads):
    """TF32 mode runs 9 to 16 rows on the tensor-core kernel (one 128-row
    tile, rows past M filled with zeros by TMA), with K split when K is long:
    every epilogue kind, ragged N, against the oracle at the TF32 tolerance,
    and the same bits through the row-streamed executor."""
    N, K = NK
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    bias = datagen.normal((N,), 8, 0.0, 0.5)
    odd = datagen.uniform((13,), 9)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_ADD, hg.input_node(odd)), (OP_RELU, None),
                          (OP_ADD, hg.input_node(bias))])
    got = run_execute(lib, gpu_ctx, root, TF32)
    want = bindings.fused_oracle(A, B, [("add", C), ("add", odd), ("relu",), ("add", bias)], threads=host_threads)
    check(got, want, TF32, f"few rows M={M} {NK}")


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("mnk", [(33, 47, 129), (100, 100, 300), (64, 1000, 5), (128, 128, 128), (200, 96, 1000)])
def test_tiny_path(lib, gpu_ctx, mnk, precision, monkeypatch, host_threads):
    """The one-launch CUDA-core kernel for tiny problems (3xTF32 mode up to
    M*N*K = 2^26; forced here in both modes with MINIXLA_TINY_MAX_MNK):
    ragged tiles, K not a multiple of the staged chunk, every epilogue kind,
    against the oracle at the 3xTF32 tolerance (fp32 FMAs)."""
    monkeypatch.setenv("MINIXLA_TINY_MAX_MNK", str(1 << 40))
    M, N, K = mnk
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    bias = datagen.normal((N,), 8, 0.0, 0.5)
    odd = datagen.uniform((13,), 9)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_ADD, hg.input_node(odd)), (OP_RELU, None),
                          (OP_ADD, hg.input_node(bias))])
    got = run_execute(lib, gpu_ctx, root, precision)
    want = bindings.fused_oracle(A, B, [("add", C), ("add", odd), ("relu",), ("add", bias)], threads=host_threads)
    check(got, want, X3, f"tiny {mnk}")


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
def test_wide_dag_on_several_streams(lib, gpu_ctx, precision):
    """Six independent branches from one input (spread over the executor's
    streams), joined by standalone adds and a final fused node: exercises
    the cross-stream waits and the release-after-all-consumers rule."""
    M, K, N = 96, 200, 136
    X = datagen.uniform((M, K), 40)
    Ws = [datagen.normal((K, N), 41 + i, 0.0, 1.0 / np.sqrt(K)) for i in range(6)]
    bs = [datagen.normal((N,), 51 + i, 0.0, 0.1) for i in range(6)]
    V = datagen.normal((N, N), 60, 0.0, 1.0 / np.sqrt(N))
    hg = HostGraph()
    x = hg.input_node(X)
    hs = [hg.fused_node(x, hg.input_node(W), [(OP_ADD, hg.input_node(b)), (OP_RELU, None)]) for W, b in zip(Ws, bs)]
    acc = hs[0]
    for h in hs[1:]:
        acc = hg.g_add(acc, h)
    root = hg.fused_node(acc, hg.input_node(V), [(OP_ADD, hs[2]), (OP_RELU, None)])
    got = run_execute(lib, gpu_ctx, root, precision)
    h_ref = [bindings.fused_oracle(X, W, [("add", b), ("relu",)]) for W, b in zip(Ws, bs)]
    a_ref = h_ref[0]
    for h in h_ref[1:]:
        a_ref = bindings.add_oracle(a_ref, h)
    want = bindings.fused_oracle(a_ref, V, [("add", h_ref[2]), ("relu",)])
    check(got, want, precision, "wide DAG", depth=2)
    again = run_execute(lib, gpu_ctx, root, precision)
    assert np.array_equal(got, again)


@pytest.mark.parametrize("chunks", ["1", "8"], ids=["one_stream", "row_streamed"])
def test_staged_host_copies(lib, gpu_ctx, chunks, monkeypatch):
    """Pageable host buffers above 2 MiB travel through the context's pinned
    staging slots (several host threads fill a slot while the previous one
    is on the link).  Results, into a library-made tensor and into a caller
    buffer, equal those of the driver's own pageable copies
    (MINIXLA_STAGED_COPY=0) bit for bit, on sizes that end mid-slot."""
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", chunks)
    M, N, K = 1531, 1536, 1540  # 9-9.4 MB operands: one full 8 MiB slot and a partial one
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(C)), (OP_RELU, None)])
    staged = run_execute(lib, gpu_ctx, root, TF32)
    into = np.zeros((M, N), np.float32)
    assert lib.gpu_execute_into(root, gpu_ctx, hg.tensor(into)) == 0, mlib.last_error()
    monkeypatch.setenv("MINIXLA_STAGED_COPY", "0")
    plain = run_execute(lib, gpu_ctx, root, TF32)
    assert np.array_equal(staged, plain)
    assert np.array_equal(into, plain)
    rows = _sample_rows(M, 64)
    want = bindings.fused_oracle(A, B, [("add", C), ("relu",)], rows=rows)
    check(staged[rows], want, TF32, "staged copies")


def test_resident_weights(lib, gpu_ctx):
    """gpu_ctx_keep_resident: the kept copy is read instead of the host data
    (so a change to the host data is not seen until release + keep), results
    match the uploading path, a moved data pointer falls back to uploading,
    and release restores plain behaviour.  Covers the streamed executor
    (M >= 256) and the one-stream executor (M < 256)."""
    import ctypes as C

    for M in (512, 64):
        N, K = 384, 256
        A, B, Cm = _relu_abc(M, N, K, c_normal=True)
        hg = HostGraph()
        bnode = hg.input_node(B)
        root = hg.fused_node(hg.input_node(A), bnode, [(OP_ADD, hg.input_node(Cm)), (OP_RELU, None)])
        plain = run_execute(lib, gpu_ctx, root, X3)
        bt = bnode.contents.output
        assert lib.gpu_ctx_keep_resident(gpu_ctx, bt) == 0
        assert np.array_equal(run_execute(lib, gpu_ctx, root, X3), plain)
        B[:] = 0.0  # host data changes in place: the resident copy is still read
        assert np.array_equal(run_execute(lib, gpu_ctx, root, X3), plain)
        assert lib.gpu_ctx_keep_resident(gpu_ctx, bt) == 0  # keep again: picks up the change
        zero = run_execute(lib, gpu_ctx, root, X3)
        np.testing.assert_array_equal(zero, np.maximum(Cm, 0))
        B2 = np.ascontiguousarray(_relu_abc(M, N, K, c_normal=True)[1])
        bt.contents.data = C.cast(C.c_void_p(B2.ctypes.data), C.POINTER(C.c_float))  # moved data: uploaded
        np.testing.assert_array_equal(run_execute(lib, gpu_ctx, root, X3), plain)
        assert lib.gpu_ctx_release_resident(gpu_ctx, None) == 0
        np.testing.assert_array_equal(run_execute(lib, gpu_ctx, root, X3), plain)


# ---------------------------------------------------------------- bare matmul fused into its consumer


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("M,H", [(8, 256), (200, 256), (1000, 256), (4096, 256), (1024, 2048)])
def test_product_fusion_in_graphs(lib, gpu_ctx, M, H, precision, monkeypatch, host_threads):
    """Config 4's pattern, y = relu(h W2 + b2) + h W2' with h W2' a bare
    matmul read only by y: both products run in one kernel (TF32 always,
    3xTF32 when its 256 x 128 pair tiles fill a quarter of the SMs, here
    (1024, 2048)).  The result matches the two-launch form
    (MINIXLA_DUAL_GEMM=0) bit for bit and the oracle within the mode's
    tolerance; M = 8 keeps the two-launch form, M = 200 runs on the
    one-stream executor, larger M row-streamed."""
    D = 96
    X = datagen.uniform((M, D), 80)
    W1 = datagen.normal((D, H), 81, 0.0, 1.0 / np.sqrt(D))
    W2 = datagen.normal((H, H), 82, 0.0, 1.0 / np.sqrt(H))
    W2p = datagen.normal((H, H), 83, 0.0, 1.0 / np.sqrt(H))
    b1 = datagen.normal((H,), 84, 0.0, 0.1)
    b2 = datagen.normal((H,), 85, 0.0, 0.1)
    hg = HostGraph()
    x = hg.input_node(X)
    h = hg.fused_node(x, hg.input_node(W1), [(OP_ADD, hg.input_node(b1)), (OP_RELU, None)])
    hw = hg.g_matmul(h, hg.input_node(W2p))
    root = hg.fused_node(h, hg.input_node(W2), [(OP_ADD, hg.input_node(b2)), (OP_RELU, None), (OP_ADD, hw)])
    fused = run_execute(lib, gpu_ctx, root, precision)
    monkeypatch.setenv("MINIXLA_DUAL_GEMM", "0")
    two = run_execute(lib, gpu_ctx, root, precision)
    monkeypatch.delenv("MINIXLA_DUAL_GEMM")
    assert np.array_equal(fused, two)
    h_ref = bindings.fused_oracle(X, W1, [("add", b1), ("relu",)], threads=host_threads)
    hw_ref = bindings.fused_oracle(h_ref, W2p, [], threads=host_threads)
    want = bindings.fused_oracle(h_ref, W2, [("add", b2), ("relu",), ("add", hw_ref)], threads=host_threads)
    check(fused, want, precision, f"product fusion M={M} H={H}", depth=2)


@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("mnkk", [(256, 256, 32, 64), (300, 520, 100, 36), (1000, 1000, 1000, 1000),
                                  (2048, 2048, 2048, 1024), (12, 260, 128, 96), (4096, 4096, 4096, 4096)])
@pytest.mark.parametrize("shared", [True, False], ids=["shared_A", "own_A2"])
def test_fused_gemm2_device_api(lib, gpu_ctx, mnkk, precision, shared, host_threads):
    """mxb_fused_gemm2: epi(A B) with a second product A2 B2 added at its
    step, against the oracle (the second product evaluated separately, as
    eval_fused adds a stored matmul).  shared_A passes A itself as A2 (the
    one-kernel form in TF32 mode); own_A2 a separate matrix (two launches)."""
    import torch

    M, N, K, K2 = mnkk
    if shared:
        K2 = K
    elif M * N * K > 2048 ** 3:
        pytest.skip("the two-launch form is covered at the smaller shapes")
    A = datagen.uniform((M, K), 90)
    B = datagen.uniform((K, N), 91)
    A2 = A if shared else datagen.uniform((M, K2), 92)
    B2 = datagen.uniform((K2, N), 93)
    bias = datagen.normal((N,), 94, 0.0, 0.5)
    dA, dB, dA2, dB2, dbias = (torch.from_numpy(x).cuda() for x in (A, B, A2, B2, bias))
    if shared:
        dA2 = dA
    out = torch.empty((M, N), device="cuda")
    steps = (mlib.EpStepDev * 3)()
    steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, dbias.data_ptr(), N, 0.0, 0)
    steps[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
    steps[2] = mlib.EpStepDev(mlib.MXB_EP_ADD_PRODUCT, 0, None, 0, 0.0, 0)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mxb_fused_gemm2(gpu_ctx, dA.data_ptr(), K, dB.data_ptr(), N, dA2.data_ptr(), K2, dB2.data_ptr(), N, K2,
                             out.data_ptr(), N, M, N, K, steps, 3, precision, stream)
    assert rc == 0, mlib.last_error()
    torch.cuda.synchronize()
    assert lib.mxb_check_device_error(gpu_ctx) == 0
    rows = None if M * N * K <= 2048 ** 3 else _sample_rows(M, 256)
    p_ref = bindings.fused_oracle(A2, B2, [], rows=rows, threads=host_threads)
    if rows is not None:  # the add operand is indexed by global row: place the sampled rows
        full = np.zeros((M, N), np.float32)
        full[rows] = p_ref
        p_ref = full
    want = bindings.fused_oracle(A, B, [("add", bias), ("relu",), ("add", p_ref)], rows=rows, threads=host_threads)
    got = out.cpu().numpy()
    check(got if rows is None else got[rows], want, precision, f"gemm2 {mnkk}", depth=2)


def test_fused_gemm2_rejects_bad_arguments(lib, gpu_ctx):
    import torch

    M, N, K = 256, 256, 64
    t = torch.zeros((M, max(N, K) + 4), device="cuda")
    out = torch.empty((M, N), device="cuda")
    p = t.data_ptr()
    relu = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
    prod = mlib.EpStepDev(mlib.MXB_EP_ADD_PRODUCT, 0, None, 0, 0.0, 0)

    def call(steps, lda2=K, a2=p):
        arr = (mlib.EpStepDev * len(steps))(*steps)
        return lib.mxb_fused_gemm2(gpu_ctx, p, K, p, N, a2, lda2, p, N, K, out.data_ptr(), N, M, N, K, arr,
                                   len(steps), TF32, None)

    assert call([relu]) == mlib.MXB_E_ARG                 # no ADD_PRODUCT step
    assert call([prod, relu, prod]) == mlib.MXB_E_ARG     # two
    assert call([prod], lda2=K + 2) == mlib.MXB_E_ARG     # row pitch not a multiple of 4
    assert call([prod], a2=p + 4) == mlib.MXB_E_ARG       # base not 16-byte aligned
    steps = (mlib.EpStepDev * 1)(prod)
    assert lib.mxb_fused_gemm(gpu_ctx, p, K, p, N, out.data_ptr(), N, M, N, K, steps, 1, TF32,
                              None) == mlib.MXB_E_ARG  # mxb_fused_gemm has no second product


# ---------------------------------------------------------------- device-pointer API


def test_device_pointer_api_matches_torch(lib, gpu_ctx):
    import torch

    M, N, K = 384, 520, 200
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    bias = torch.randn(N, device="cuda", generator=g)
    out = torch.empty(M, N, device="cuda")
    steps = (mlib.EpStepDev * 3)()
    steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, bias.data_ptr(), N, 0.0, 0)
    steps[1] = mlib.EpStepDev(mlib.MXB_EP_SCALE, 0, None, 0, 0.5, 0)
    steps[2] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.mxb_fused_gemm(gpu_ctx, A.data_ptr(), K, B.data_ptr(), N, out.data_ptr(), N, M, N, K, steps, 3,
                            X3, stream)
    assert rc == 0, mlib.last_error()
    torch.cuda.synchronize()
    ref = torch.relu((A.double() @ B.double() + bias.double()) * 0.5)
    assert rel_frobenius(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5


def test_device_api_from_several_threads(lib, gpu_ctx):
    """The device-pointer launches may share one context across host threads
    (its pool is locked): four threads, each on its own stream, run the
    3xTF32 GEMM (which takes pooled workspace) and get the single-threaded
    results bit for bit."""
    import threading

    import torch

    M, N, K = 512, 384, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.rand(M, K, device="cuda", generator=g) - 0.5
    B = torch.rand(K, N, device="cuda", generator=g) - 0.5
    steps = (mlib.EpStepDev * 1)()
    steps[0] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
    want = torch.empty(M, N, device="cuda")
    assert lib.mxb_fused_gemm(gpu_ctx, A.data_ptr(), K, B.data_ptr(), N, want.data_ptr(), N, M, N, K, steps, 1, X3,
                              None) == 0
    assert lib.mxb_check_device_error(gpu_ctx) == 0
    outs = [torch.empty(M, N, device="cuda") for _ in range(4)]
    streams = [torch.cuda.Stream() for _ in range(4)]
    errors = []

    def work(i):
        for _ in range(20):
            rc = lib.mxb_fused_gemm(gpu_ctx, A.data_ptr(), K, B.data_ptr(), N, outs[i].data_ptr(), N, M, N, K, steps,
                                    1, X3, streams[i].cuda_stream)
            if rc != 0:
                errors.append(mlib.last_error())
                return

    threads = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    assert lib.mxb_check_device_error(gpu_ctx) == 0
    for o in outs:
        assert torch.equal(o, want)


def test_standalone_elementwise_device_api(lib, gpu_ctx):
    import torch

    n = 3 * 1024 * 1024 + 3
    x = torch.randn(n, device="cuda")
    b = torch.randn(1024 * 3 + 1, device="cuda")
    a = torch.randn((1024 * 3 + 1) * 7, device="cuda")
    out = torch.empty_like(x)
    assert lib.mxb_relu(gpu_ctx, x.data_ptr(), n, out.data_ptr(), None) == 0
    lib.mxb_check_device_error(gpu_ctx)
    assert torch.equal(out, torch.where(x > 0, x, torch.zeros_like(x)))
    out2 = torch.empty_like(a)
    assert lib.mxb_add(gpu_ctx, a.data_ptr(), a.numel(), b.data_ptr(), b.numel(), out2.data_ptr(), None) == 0
    lib.mxb_check_device_error(gpu_ctx)
    assert torch.equal(out2, a + b.repeat(7))


# ---------------------------------------------------------------- failure paths (no GPU fault)


def test_bounded_wait_times_out_cleanly(lib, gpu_ctx, golden):
    """A kernel waiting on a barrier nothing completes gives up after its limit,
    reports MXB_E_TIMEOUT, and the context keeps working."""
    rc = lib.mxb_selftest_wait_timeout(gpu_ctx, 2_000_000)  # 2 ms
    assert rc == mlib.MXB_E_TIMEOUT
    assert lib.mxb_check_device_error(gpu_ctx) == 0
    case = next(c for c in CASES if c[0] == "config1_128")
    hg, root = host_graph(case[1], case[2])
    check(run_execute(lib, gpu_ctx, root, X3), golden["config1_128:__out__"], X3)


def test_unsupported_ops_fail_loudly(lib, gpu_ctx):
    hg = HostGraph()
    a = hg.input_node(np.ones((2, 2), np.float32))
    mul = hg._node(OP_MUL, [a, a])
    assert not lib.gpu_execute(mul, gpu_ctx)
    assert "not supported" in mlib.last_error()
    bad = hg.fused_node(hg.input_node(np.ones((2, 3), np.float32)), hg.input_node(np.ones((2, 3), np.float32)), [])
    assert not lib.gpu_execute(bad, gpu_ctx)
    assert "incompatible" in mlib.last_error()
    bad_add = hg.g_add(hg.input_node(np.ones((2, 3), np.float32)), hg.input_node(np.ones((2,), np.float32)))
    assert not lib.gpu_execute(bad_add, gpu_ctx)


# Allocation order of the first call: A, B, C, out, then the two 3xTF32 low-part buffers.
_OOM_CHILD = r"""
import sys, numpy as np
sys.path.insert(0, sys.argv[1])
import torch
from minixla_b200 import lib as mlib
from minixla_b200.abi import HostGraph, OP_ADD, OP_RELU, free_host_tensor
lib = mlib.load()
hg = HostGraph()
A = np.ones((300, 200), np.float32); B = np.ones((200, 100), np.float32); Cm = np.ones((300, 100), np.float32)
root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(Cm)), (OP_RELU, None)])
ctx = lib.gpu_ctx_create()
torch.cuda.init()
free0 = torch.cuda.mem_get_info(0)[0]
t = lib.gpu_execute(root, ctx)
assert not t, "allocation failure must give NULL"
assert "MINIXLA_FAIL_ALLOC_AT" in mlib.last_error()
t = lib.gpu_execute(root, ctx)          # the next call succeeds on the same context
assert t
free_host_tensor(t)
lib.gpu_ctx_destroy(ctx)
assert torch.cuda.mem_get_info(0)[0] >= free0 - 16 * 2**20
print("OK")
"""


@pytest.mark.parametrize("fail_at", [1, 3, 4, 5, 6])
def test_allocation_failure_injection(fail_at):
    # The tensor-core path (not the tiny-problem kernel) so the graph makes its full set of
    # allocations: inputs, output and the 3xTF32 low parts.
    env = dict(os.environ, MINIXLA_FAIL_ALLOC_AT=str(fail_at), MINIXLA_TINY_MAX_MNK="0")
    r = subprocess.run([sys.executable, "-c", _OOM_CHILD, str(ROOT)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


# (M, N, K) whose TF32 CTA-pair tiles do not fill a whole number of waves on
# 74 pairs: 320 tiles of 256 x 256 (98 stream-K), 312 of them with a ragged
# M, N and K (90 stream-K), and the 8-way split of config 5 (256 wide tiles of
# 256 x 512: 148 run whole, 108 stream-K), so both tile widths hand off.
STREAMK_SHAPES = [(5120, 4096, 2048), (3300, 6001, 2049), (4096, 8192, 8192)]


@pytest.mark.parametrize("mnk", STREAMK_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in STREAMK_SHAPES])
def test_stream_k_keeps_the_bits(lib, gpu_ctx, mnk, monkeypatch, host_threads):
    """Stream-K hands a split tile's raw fp32 accumulator from one CTA pair to
    the next and continues the same MMA chain, so the output must be bit-equal
    to the launch that runs every tile whole (MINIXLA_STREAMK=0) -- and match
    the oracle on sampled rows (tile edges, shard-like edges, random rows)
    within the TF32 tolerance, for relu(A.B + C) + bias."""
    import torch

    M, N, K = mnk
    sms = torch.cuda.get_device_properties(lib.gpu_ctx_device(gpu_ctx)).multi_processor_count
    plan = mlib.gemm_plan(M, N, K, TF32, sms)
    if plan.kernel != mlib.MXB_KERNEL_CTA_PAIR or plan.streamk_tiles == 0:
        pytest.skip(f"{sms} SMs: {mnk} runs no stream-K tail")
    dev = torch.device("cuda", lib.gpu_ctx_device(gpu_ctx))
    A_h = datagen.uniform((M, K), 30)
    B_h = datagen.uniform((K, N), 31)
    C_h = datagen.normal((M, N), 32)
    bias_h = datagen.normal((N,), 33, 0.0, 0.5)
    Kp, Np = (K + 3) // 4 * 4, (N + 3) // 4 * 4

    def padded(x, cols):
        t = torch.zeros((x.shape[0], cols), device=dev)
        t[:, :x.shape[1]] = torch.from_numpy(x).to(dev)
        return t

    A, B = padded(A_h, Kp), padded(B_h, Np)
    C = torch.from_numpy(C_h).to(dev)
    bias = torch.from_numpy(bias_h).to(dev)
    steps = (mlib.EpStepDev * 3)()
    steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, C.data_ptr(), N, 0.0, 0)
    steps[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
    steps[2] = mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, bias.data_ptr(), N, 0.0, 0)
    outs = {}
    for sk in ("1", "0"):
        monkeypatch.setenv("MINIXLA_STREAMK", sk)
        out = torch.full((M, N), float("nan"), device=dev)
        for _ in range(2):  # twice: flags and accumulators of one launch do not leak into the next
            rc = lib.mxb_fused_gemm(gpu_ctx, A.data_ptr(), Kp, B.data_ptr(), Np, out.data_ptr(), N, M, N, K,
                                    steps, 3, TF32, None)
            assert rc == 0, mlib.last_error()
        assert lib.mxb_check_device_error(gpu_ctx) == 0
        outs[sk] = out.cpu().numpy()
    assert not np.isnan(outs["1"]).any()
    assert np.array_equal(outs["1"], outs["0"]), "stream-K changed the bits"
    rng = np.random.default_rng(M + N)
    rows = sorted({0, 1, 127, 128, 255, 256, 257, M // 2, M - 2, M - 1, *rng.integers(0, M, 48).tolist()})
    want = bindings.fused_oracle(A_h, B_h, [("add", C_h), ("relu",), ("add", bias_h)], rows=rows, threads=host_threads)
    check(outs["1"][rows], want, TF32, f"stream-K {mnk}")


@pytest.mark.parametrize("variant", ["pair512", "pair"])
@pytest.mark.parametrize("mnk", [(300, 520, 100), (2047, 1030, 1500), (8000, 8000, 512)])
def test_box_epilogue_keeps_the_bits(lib, gpu_ctx, mnk, variant, monkeypatch, host_threads):
    """The TF32 CTA-pair kernels read C and write the output as 32 x 32 TMA
    boxes through shared memory (rows past M and columns past N zero-filled on
    the way in, clipped on the way out).  The result must be bit-equal to the
    per-lane form (MINIXLA_EPI_TMA=0) on partial row, column and k tiles,
    including a second FULL add (loaded per lane) and a bias row after relu,
    and match the oracle within the TF32 tolerance."""
    monkeypatch.setenv("MINIXLA_GEMM_VARIANT", variant)
    M, N, K = mnk
    A, B, C = _relu_abc(M, N, K, c_normal=True)
    C2 = datagen.uniform((M, N), 41)
    bias = datagen.normal((N,), 42, 0.0, 0.5)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_ADD, hg.input_node(C2)), (OP_RELU, None),
                          (OP_ADD, hg.input_node(bias))])
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "1")
    boxed = run_execute(lib, gpu_ctx, root, TF32)
    monkeypatch.setenv("MINIXLA_EPI_TMA", "0")
    per_lane = run_execute(lib, gpu_ctx, root, TF32)
    assert np.array_equal(boxed, per_lane), "the box epilogue changed the bits"
    rows = sorted({0, 1, 255, 256, M // 2, M - 2, M - 1, *np.random.default_rng(M).integers(0, M, 24).tolist()})
    want = bindings.fused_oracle(A, B, [("add", C), ("add", C2), ("relu",), ("add", bias)], rows=rows,
                                 threads=host_threads)
    check(boxed[rows], want, TF32, f"box epilogue {variant} {mnk}")


@pytest.mark.parametrize("variant", ["pair512", "pair"])
def test_box_epilogue_output_only(lib, gpu_ctx, variant, monkeypatch, host_threads):
    """A node whose first epilogue step is not a full add (a bias row, then
    relu) writes through the output boxes alone.  With 8192 x 1120 outputs
    each warp runs several tiles and the last column tile has an odd number
    of 32-column chunks, so a tile may start on the box its predecessor's
    last store is still reading: bit-equal to the per-lane form and within
    the TF32 tolerance of the oracle."""
    monkeypatch.setenv("MINIXLA_GEMM_VARIANT", variant)
    M, N, K = 8192, 1120, 256
    A, B, _ = _relu_abc(M, N, K, c_normal=True)
    bias = datagen.normal((N,), 43, 0.0, 0.5)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(bias)), (OP_RELU, None)])
    monkeypatch.setenv("MINIXLA_STREAM_CHUNKS", "1")
    boxed = run_execute(lib, gpu_ctx, root, TF32)
    monkeypatch.setenv("MINIXLA_EPI_TMA", "0")
    per_lane = run_execute(lib, gpu_ctx, root, TF32)
    assert np.array_equal(boxed, per_lane), "the output boxes changed the bits"
    rows = sorted({0, 255, 256, 4095, 4096, M - 1, *np.random.default_rng(7).integers(0, M, 24).tolist()})
    want = bindings.fused_oracle(A, B, [("add", bias), ("relu",)], rows=rows, threads=host_threads)
    check(boxed[rows], want, TF32, f"output boxes {variant}")
