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


def test_noalloc_matches_pooled_entry_point_twice(lib, gpu_ctx):
    import torch

    dev = torch.device("cuda", lib.gpu_ctx_device(gpu_ctx))
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(dev)
    g = torch.Generator(device=dev).manual_seed(1234)
    shapes = [(640, 528, 1000), (1000, 264, 1024)]  # (M, N, K): M*K + K*N within the 4 Mi-float array
    for call, (M, N, K) in enumerate(shapes):
        A = torch.rand(M, K, device=dev, generator=g) * 2 - 1
        B = torch.rand(K, N, device=dev, generator=g) * 2 - 1
        C = torch.randn(M, N, device=dev, generator=g)
        bias = torch.randn(N, device=dev, generator=g)
        steps, n = _steps([
            mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, C.data_ptr(), N, 0.0, 0),
            mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0),
            mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, bias.data_ptr(), N, 0.0, 0),
        ])
        out_pool = torch.full((M, N), float("nan"), device=dev)
        out_none = torch.full((M, N), float("nan"), device=dev)
        torch.cuda.synchronize()
        rc = lib.mxb_fused_gemm(gpu_ctx, A.data_ptr(), K, B.data_ptr(), N, out_pool.data_ptr(), N, M, N, K,
                                steps, n, mlib.GPU_PRECISION_3XTF32, stream.cuda_stream)
        assert rc == 0, mlib.last_error()
        assert lib.mxb_check_device_error(gpu_ctx) == 0
        rc = lib.mxb_fused_gemm_noalloc(A.data_ptr(), K, B.data_ptr(), N, out_none.data_ptr(), N, M, N, K,
                                        steps, n, stream.cuda_stream)
        assert rc == 0, f"call {call}: {mlib.last_error()}"
        torch.cuda.synchronize()
        assert not torch.isnan(out_none).any(), f"call {call}: output not fully written"
        assert _rel(out_none, out_pool) <= TOL_3XTF32, f"call {call}: differs from mxb_fused_gemm"
        want = torch.relu(A.double() @ B.double() + C.double()) + bias.double()
        assert _rel(out_none, want) <= TOL_3XTF32, f"call {call}: differs from the float64 product"


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
