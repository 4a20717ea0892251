"""Multi-GPU context (gpu_ctx_create_multi): row-sharded execution over every
visible GPU, checked against the oracle and against the one-GPU result.
Skipped where fewer than two GPUs are visible."""
import numpy as np
import pytest

from minixla_b200 import datagen
from minixla_b200 import lib as mlib
from minixla_b200.abi import OP_ADD, OP_RELU, HostGraph, free_host_tensor, tensor_to_numpy
from oracle.bindings import fused_oracle
from tests.graph_eval import rel_frobenius

pytestmark = pytest.mark.gpu

TF32, X3 = mlib.GPU_PRECISION_TF32, mlib.GPU_PRECISION_3XTF32
TOL = {TF32: 2e-3, X3: 1e-5}


def _ngpu():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


needs2 = pytest.mark.skipif(_ngpu() < 2, reason="needs at least two GPUs")


@pytest.fixture(scope="module")
def multi_ctx(lib):
    n = _ngpu()
    if n < 2:
        pytest.skip("needs at least two GPUs")
    ctx = lib.gpu_ctx_create_multi(n)
    assert ctx, mlib.last_error()
    assert lib.gpu_ctx_ngpu(ctx) == n
    yield ctx
    lib.gpu_ctx_destroy(ctx)


def _run(lib, ctx, root, precision):
    assert lib.gpu_ctx_set_precision(ctx, precision) == 0
    t = lib.gpu_execute(root, ctx)
    assert t, mlib.last_error()
    out = tensor_to_numpy(t)
    free_host_tensor(t)
    return out


@needs2
@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
@pytest.mark.parametrize("M", [1001, 4096])
def test_sharded_fused_node(lib, multi_ctx, gpu_ctx, precision, M):
    N, K = 768, 512
    A, B, C = datagen.uniform((M, K), 0), datagen.uniform((K, N), 1), datagen.normal((M, N), 2)
    bias = datagen.normal((N,), 3, 0.0, 0.5)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B),
                         [(OP_ADD, hg.input_node(C)), (OP_RELU, None), (OP_ADD, hg.input_node(bias))])
    got = _run(lib, multi_ctx, root, precision)
    want = fused_oracle(A, B, [("add", C), ("relu",), ("add", bias)])
    assert rel_frobenius(got, want) <= TOL[precision]
    one = _run(lib, gpu_ctx, root, precision)
    assert rel_frobenius(got, one) <= TOL[precision]


@needs2
def test_sharded_mlp_dag(lib, multi_ctx):
    from tests.golden.cases import case_mlp_small
    from tests.graph_eval import host_graph, oracle_eval

    name, inputs, build = case_mlp_small(M=1536, D=256, H=512)
    hg, root = host_graph(inputs, build)
    got = _run(lib, multi_ctx, root, X3)
    assert rel_frobenius(got, oracle_eval(inputs, build)) <= 3 * TOL[X3]


@needs2
@pytest.mark.parametrize("precision", [TF32, X3], ids=["tf32", "3xtf32"])
def test_intermediate_read_whole_is_all_gathered(lib, multi_ctx, precision):
    """H = relu(X W + b) is row-sharded, then read whole as the B operand of
    out = X H + V: the GPUs all-gather H's shards over NCCL first."""
    M = K = 640
    N = 384
    X = datagen.uniform((M, K), 10)
    W = datagen.normal((K, M), 11, 0.0, 1.0 / np.sqrt(K))
    b = datagen.normal((M,), 12, 0.0, 0.1)
    V = datagen.normal((M, M), 13)
    hg = HostGraph()
    x = hg.input_node(X)
    h = hg.fused_node(x, hg.input_node(W), [(OP_ADD, hg.input_node(b)), (OP_RELU, None)])
    root = hg.fused_node(x, h, [(OP_ADD, hg.input_node(V))])
    got = _run(lib, multi_ctx, root, precision)
    H = fused_oracle(X, W, [("add", b), ("relu",)])
    want = fused_oracle(X, H, [("add", V)])
    assert rel_frobenius(got, want) <= 2 * TOL[precision]


@needs2
def test_graph_that_does_not_shard_runs_on_gpu0(lib, multi_ctx):
    """An intermediate whose rows are not the root's rows (here the B operand
    of the root is computed from other operands) keeps the graph on GPU 0."""
    M, K, N, J = 300, 256, 192, 128
    X = datagen.uniform((M, K), 20)
    P = datagen.uniform((K, J), 21)
    Q = datagen.uniform((J, N), 22)
    hg = HostGraph()
    inner = hg.fused_node(hg.input_node(P), hg.input_node(Q), [(OP_RELU, None)])   # K x N, rows != M
    root = hg.fused_node(hg.input_node(X), inner, [])
    got = _run(lib, multi_ctx, root, X3)
    want = fused_oracle(X, fused_oracle(P, Q, [("relu",)]), [])
    assert rel_frobenius(got, want) <= 2 * TOL[X3]


@needs2
def test_sharded_with_resident_weight(lib, multi_ctx, gpu_ctx):
    M, N, K = 2048, 512, 384
    A, B, C = datagen.uniform((M, K), 30), datagen.uniform((K, N), 31), datagen.normal((M, N), 32)
    hg = HostGraph()
    bnode = hg.input_node(B)
    root = hg.fused_node(hg.input_node(A), bnode, [(OP_ADD, hg.input_node(C)), (OP_RELU, None)])
    plain = _run(lib, multi_ctx, root, X3)
    assert lib.gpu_ctx_keep_resident(multi_ctx, bnode.contents.output) == 0
    kept = _run(lib, multi_ctx, root, X3)
    assert lib.gpu_ctx_release_resident(multi_ctx, None) == 0
    assert np.array_equal(plain, kept)
    assert rel_frobenius(kept, fused_oracle(A, B, [("add", C), ("relu",)])) <= TOL[X3]
