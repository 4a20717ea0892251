"""GPU test of mxb_fused_gemm_noalloc, the entry point for callers that
cannot allocate device memory (for example a plugin living inside a framework
that owns the device-memory budget, or a serving loop that must not take the
device-wide synchronisation of cudaMalloc).  Its low-part scratch is a fixed
array inside the library, so the test checks that two calls in a row -- the
second reusing the array the first one filled -- both match the pooled
entry point mxb_fused_gemm, and that a problem too large for the array is
refused with an error instead of running.

The file name sorts last so a run that stops at the first failure has already
run every other test."""
import numpy as np
import pytest

from minixla_b200 import lib as mlib

pytestmark = pytest.mark.gpu

TOL_3XTF32 = 1e-5


def _steps(kinds):
    arr = (mlib.EpStepDev * max(1, len(kinds)))()
    for i, k in enumerate(kinds):
        arr[i] = k
    return arr, len(kinds)


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


# (M, N, K, extra output pitch): M*K + K*N within the 4 Mi-float array.  One
# and sixteen rows (which the pooled entry point sends to its few-row kernel),
# the single-CTA tiles, an odd output pitch, and 2048 x 2048 x 1024, which
# fills the array exactly and runs on the CTA-pair kernel.
SHAPES = [(1, 528, 1000, 0), (16, 528, 1000, 0), (640, 528, 1000, 0), (1000, 264, 1024, 3),
          (2048, 2048, 1024, 0)]


@pytest.mark.parametrize("M,N,K,pad", SHAPES, ids=[f"{m}x{n}x{k}" + ("_odd_ldo" if p else "")
                                                  for m, n, k, p in SHAPES])
def test_noalloc_matches_pooled_entry_point_twice(lib, gpu_ctx, M, N, K, pad):
    """Two calls in a row on the same inputs: each matches mxb_fused_gemm and
    the float64 product within the 3xTF32 tolerance, the two are bit-equal
    (the second reuses the array the first filled), the columns past N of a
    wider output pitch are never written, and the second call leaves the
    device's free memory unchanged (the first may still load kernels)."""
    import torch

    dev = torch.device("cuda", lib.gpu_ctx_device(gpu_ctx))
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    g = torch.Generator(device=dev).manual_seed(1234 + M)
    ldo = N + pad
    A = torch.rand(M, K, device=dev, generator=g) * 2 - 1
    B = torch.rand(K, N, device=dev, generator=g) * 2 - 1
    C = torch.randn(M, N, device=dev, generator=g)
    bias = torch.randn(N, device=dev, generator=g)
    steps, n = _steps([
        mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, C.data_ptr(), N, 0.0, 0),
        mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0),
        mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, bias.data_ptr(), N, 0.0, 0),
    ])
    if M == 2048:
        plan = mlib.gemm_plan(M, N, K, mlib.GPU_PRECISION_3XTF32,
                              torch.cuda.get_device_properties(dev).multi_processor_count)
        assert plan.kernel == mlib.MXB_KERNEL_CTA_PAIR, "2048 x 2048 x 1024 should run on the CTA-pair kernel"
    out_pool = torch.full((M, N), float("nan"), device=dev)
    torch.cuda.synchronize()
    rc = lib.mxb_fused_gemm(gpu_ctx, A.data_ptr(), K, B.data_ptr(), N, out_pool.data_ptr(), N, M, N, K,
                            steps, n, mlib.GPU_PRECISION_3XTF32, stream.cuda_stream)
    assert rc == 0, mlib.last_error()
    assert lib.mxb_check_device_error(gpu_ctx) == 0
    want = torch.relu(A.double() @ B.double() + C.double()) + bias.double()
    results = []
    for call in range(2):
        out = torch.full((M, ldo), float("nan"), device=dev)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        rc = lib.mxb_fused_gemm_noalloc(A.data_ptr(), K, B.data_ptr(), N, out.data_ptr(), ldo, M, N, K,
                                        steps, n, stream.cuda_stream)
        assert rc == 0, f"call {call}: {mlib.last_error()}"
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info(dev)[0] == free_before, "the second call changed free device memory"
        got = out[:, :N]
        assert not torch.isnan(got).any(), f"call {call}: output not fully written"
        if pad:
            assert torch.isnan(out[:, N:]).all(), f"call {call}: wrote past column N of the output rows"
        assert _rel(got, out_pool) <= TOL_3XTF32, f"call {call}: differs from mxb_fused_gemm"
        assert _rel(got, want) <= TOL_3XTF32, f"call {call}: differs from the float64 product"
        results.append(got.clone())
    assert torch.equal(results[0], results[1]), "two calls on the same inputs gave different bits"


def test_noalloc_refuses_a_capturing_stream(lib, gpu_ctx):
    """The call reads its error word back and synchronises its stream, which
    a stream capture does not allow: on a capturing stream it returns
    MXB_E_ARG without enqueuing anything, and the caller's capture survives."""
    import torch

    dev = torch.device("cuda", lib.gpu_ctx_device(gpu_ctx))
    torch.cuda.set_device(dev)
    M, N, K = 128, 128, 128
    A = torch.rand(M, K, device=dev)
    B = torch.rand(K, N, device=dev)
    out = torch.zeros(M, N, device=dev)
    stream = torch.cuda.Stream(dev)
    # set-up call outside any capture
    assert lib.mxb_fused_gemm_noalloc(A.data_ptr(), K, B.data_ptr(), N, out.data_ptr(), N, M, N, K, None, 0,
                                      stream.cuda_stream) == 0, mlib.last_error()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        rc = lib.mxb_fused_gemm_noalloc(A.data_ptr(), K, B.data_ptr(), N, out.data_ptr(), N, M, N, K, None, 0,
                                        stream.cuda_stream)
        out.add_(1.0)  # the capture is still usable after the refusal
    assert rc == mlib.MXB_E_ARG
    assert "captured" in mlib.last_error()
    want = out + 1.0
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    del graph


def test_noalloc_refuses_problems_beyond_its_array(lib, gpu_ctx):
    import torch

    dev = torch.device("cuda", lib.gpu_ctx_device(gpu_ctx))
    M = N = K = 2048  # M*K + K*N = 8 Mi floats > 4 Mi
    A = torch.zeros(M, K, device=dev)
    B = torch.zeros(K, N, device=dev)
    out = torch.zeros(M, N, device=dev)
    rc = lib.mxb_fused_gemm_noalloc(A.data_ptr(), K, B.data_ptr(), N, out.data_ptr(), N, M, N, K, None, 0, None)
    assert rc == mlib.MXB_E_ARG
    assert "scratch" in mlib.last_error()
