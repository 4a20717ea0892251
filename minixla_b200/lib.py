"""Loads libminixla_b200.so and declares its C ABI for ctypes callers.

There is no fallback: if the native library is missing or cannot be loaded,
``load()`` raises.  Every entry point prototype matches
``include/minixla_b200.h``.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

from .abi import Node, Tensor

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libminixla_b200.so"

GPU_PRECISION_TF32 = 1
GPU_PRECISION_3XTF32 = 3

MXB_EP_ADD_FULL, MXB_EP_ADD_ROW, MXB_EP_ADD_MOD, MXB_EP_RELU, MXB_EP_SCALE, MXB_EP_ADD_PRODUCT = range(6)
MXB_OK, MXB_E_ARG, MXB_E_CUDA, MXB_E_NOMEM, MXB_E_TIMEOUT, MXB_E_UNSUPPORTED = 0, -1, -2, -3, -4, -5
MXB_MAX_EPILOGUE = 16
MXB_MAX_PEERS = 7
MXB_IPC_HANDLE_BYTES = 64

# Every symbol the header declares, with (restype, argtypes).
PROTOTYPES = {
    "gpu_ctx_create": (C.c_void_p, []),
    "gpu_ctx_create_on": (C.c_void_p, [C.c_int]),
    "gpu_ctx_create_multi": (C.c_void_p, [C.c_int]),
    "gpu_ctx_ngpu": (C.c_int, [C.c_void_p]),
    "gpu_ctx_keep_resident": (C.c_int, [C.c_void_p, C.POINTER(Tensor)]),
    "gpu_ctx_release_resident": (C.c_int, [C.c_void_p, C.POINTER(Tensor)]),
    "mxb_shard_rows": (C.c_int, [C.c_longlong, C.c_int, C.c_int, C.POINTER(C.c_longlong), C.POINTER(C.c_longlong)]),
    "gpu_ctx_destroy": (None, [C.c_void_p]),
    "gpu_execute": (C.POINTER(Tensor), [C.POINTER(Node), C.c_void_p]),
    "gpu_execute_into": (C.c_int, [C.POINTER(Node), C.c_void_p, C.POINTER(Tensor)]),
    "gpu_time_kernel_ms": (C.c_double, [C.POINTER(Node), C.c_void_p, C.c_int, C.c_int]),
    "gpu_run_tensorcore": (C.POINTER(Tensor), [C.POINTER(Node), C.c_void_p]),
    "gpu_time_kernel_tc_ms": (C.c_double, [C.POINTER(Node), C.c_void_p, C.c_int, C.c_int]),
    "gpu_run_fused": (C.POINTER(Tensor), [C.POINTER(Node), C.c_char_p]),
    "gpu_ctx_set_precision": (C.c_int, [C.c_void_p, C.c_int]),
    "gpu_ctx_get_precision": (C.c_int, [C.c_void_p]),
    "gpu_ctx_device": (C.c_int, [C.c_void_p]),
    "mxb_fused_gemm": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong,
         C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p],
    ),
    "mxb_fused_gemm2": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p,
         C.c_longlong, C.c_int, C.c_void_p, C.c_longlong, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int,
         C.c_void_p],
    ),
    "mxb_fused_gemm_noalloc": (
        C.c_int,
        [C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong,
         C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p],
    ),
    "mxb_fused_gemm_allgather": (
        C.c_int,
        [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong,
         C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p],
    ),
    "mxb_ipc_alloc": (C.c_int, [C.c_int, C.c_size_t, C.POINTER(C.c_void_p), C.POINTER(C.c_ubyte)]),
    "mxb_ipc_open": (C.c_int, [C.c_int, C.POINTER(C.c_ubyte), C.POINTER(C.c_void_p)]),
    "mxb_ipc_close": (C.c_int, [C.c_int, C.c_void_p]),
    "mxb_ipc_free": (C.c_int, [C.c_int, C.c_void_p]),
    "mxb_gather_push_count": (C.c_ulonglong, []),
    "mxb_gemm_plan_for": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "mxb_gemm_plan_batch_for": (C.c_int, [C.c_longlong, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "mxb_add": (C.c_int, [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]),
    "mxb_relu": (C.c_int, [C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]),
    "mxb_check_device_error": (C.c_int, [C.c_void_p]),
    "mxb_selftest_wait_timeout": (C.c_int, [C.c_void_p, C.c_ulonglong]),
    "mxb_launch_count": (C.c_ulonglong, []),
    "mxb_last_error": (C.c_char_p, []),
}


MXB_KERNEL_SKINNY, MXB_KERNEL_TINY, MXB_KERNEL_SINGLE_CTA, MXB_KERNEL_CTA_PAIR = 1, 2, 3, 4


class GemmPlan(C.Structure):
    """Mirror of ``mxb_gemm_plan``."""

    _fields_ = [
        ("kernel", C.c_int),
        ("tile_rows", C.c_int),
        ("tile_cols", C.c_int),
        ("k_splits", C.c_int),
        ("products", C.c_int),
        ("streamk_tiles", C.c_int),
        ("reserved", C.c_int * 2),
    ]


def gemm_plan(M: int, N: int, K: int, precision: int, num_sms: int = 148, batch: int = 0) -> GemmPlan:
    """What mxb_gemm_plan_for (batch = 0) or mxb_gemm_plan_batch_for reports
    for M x N x K products (host-only)."""
    plan = GemmPlan()
    if batch:
        rc = load().mxb_gemm_plan_batch_for(batch, M, N, K, precision, num_sms, C.byref(plan))
    else:
        rc = load().mxb_gemm_plan_for(M, N, K, precision, num_sms, C.byref(plan))
    if rc != 0:
        raise ValueError(f"mxb_gemm_plan_for: {last_error()}")
    return plan


class EpStepDev(C.Structure):
    """Mirror of ``mxb_ep_step``."""

    _fields_ = [
        ("kind", C.c_int),
        ("reserved", C.c_int),
        ("operand", C.c_void_p),
        ("ld_or_size", C.c_longlong),
        ("scale", C.c_float),
        ("reserved2", C.c_int),
    ]


assert C.sizeof(EpStepDev) == 32

_lib = None


def load() -> C.CDLL:
    """Returns the loaded native library, declaring every prototype."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("MINIXLA_B200_LIB", LIB_PATH))
    if not path.exists():
        raise RuntimeError(
            f"minixla_b200: native library {path} is missing; build it with `python -m minixla_b200.build`"
        )
    lib = C.CDLL(str(path))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return (load().mxb_last_error() or b"").decode()
