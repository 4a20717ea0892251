"""ctypes bindings for the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only tests/, the package's smoke() and bench.py's CPU-baseline leg use this
module.  It exposes:

* ``fused_oracle(...)``: the C restatement of eval_fused (fused_oracle.c),
  bit-exact with the reference in fp32, or float64 for error budgets;
* ``RefGraph``: MiniXLA's own host API (create_tensor, input_node, g_matmul,
  g_add, g_relu, fused_node, optimize, execute, free_graph -- tensor.c,
  graph.c, optimizer.c) from ``_ref/libminixla_ref.so``, compiled unmodified
  from the reference sources by ``oracle/Makefile``.  Absent where that
  library was not built; ``ref_available()`` says which.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libminixla_ref.so"

ORACLE_ADD, ORACLE_RELU, ORACLE_SCALE = 0, 1, 2


class _Step(C.Structure):
    _fields_ = [("kind", C.c_int), ("op", C.c_void_p), ("op_size", C.c_longlong), ("scale", C.c_float)]


_oracle = None
_ref = None


def oracle_lib() -> C.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            raise RuntimeError(f"{ORACLE_LIB} missing: run `make -C oracle oracle`")
        lib = C.CDLL(str(ORACLE_LIB))
        lib.oracle_fused_rows.restype = C.c_int
        lib.oracle_fused_rows.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong, C.c_longlong,
                                          C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p, C.c_int,
                                          C.c_int, C.c_int]
        lib.oracle_add.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_void_p]
        lib.oracle_relu.argtypes = [C.c_void_p, C.c_longlong, C.c_void_p]
        _oracle = lib
    return _oracle


def _steps(steps):
    keep, arr = [], (_Step * max(1, len(steps)))()
    for i, s in enumerate(steps):
        if s[0] == "add":
            op = np.ascontiguousarray(s[1], dtype=np.float32).reshape(-1)
            keep.append(op)
            arr[i] = _Step(ORACLE_ADD, op.ctypes.data, op.size, 0.0)
        elif s[0] == "relu":
            arr[i] = _Step(ORACLE_RELU, None, 0, 0.0)
        elif s[0] == "scale":
            arr[i] = _Step(ORACLE_SCALE, None, 0, float(s[1]))
        else:
            raise ValueError(s)
    return arr, keep


def fused_oracle(A: np.ndarray, B: np.ndarray, steps=(), rows=None, f64: bool = False,
                 threads: int | None = None) -> np.ndarray:
    """epi(A @ B) per eval_fused (graph.c:64-115).  steps: ("add", operand) /
    ("relu",) / ("scale", s).  rows: optional list of output rows to evaluate."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    rows = np.arange(M, dtype=np.int64) if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((len(rows), N), dtype=np.float64 if f64 else np.float32)
    arr, keep = _steps(list(steps))
    rc = oracle_lib().oracle_fused_rows(A.ctypes.data, B.ctypes.data, out.ctypes.data, M, N, K,
                                        rows.ctypes.data, len(rows), arr, len(steps), int(f64),
                                        threads or os.cpu_count() or 1)
    if rc != 0:
        raise RuntimeError("oracle_fused_rows failed")
    return out


def fused_oracle_batched(A: np.ndarray, B: np.ndarray, steps=(), f64: bool = False,
                         threads: int | None = None) -> np.ndarray:
    """Batched eval_fused (graph.c:80-113): A [..., M, K], B [..., K, N].
    Batch bt evaluates the rows bt*M .. bt*M+M-1 of A viewed as one tall
    matrix against its own B; the global row index also drives the ADD
    operands' modulo rule, exactly as eval_fused's flat index
    (bt*M*N + i*N + j) % size does."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    *batch, M, K = A.shape
    N = B.shape[-1]
    nb = int(np.prod(batch)) if batch else 1
    A2 = A.reshape(nb * M, K)
    B3 = B.reshape(nb, K, N)
    out = np.empty((nb * M, N), dtype=np.float64 if f64 else np.float32)
    arr, keep = _steps(list(steps))
    for bt in range(nb):
        rows = np.arange(bt * M, (bt + 1) * M, dtype=np.int64)
        part = np.empty((M, N), dtype=out.dtype)
        Bb = np.ascontiguousarray(B3[bt])
        rc = oracle_lib().oracle_fused_rows(A2.ctypes.data, Bb.ctypes.data, part.ctypes.data, nb * M, N, K,
                                            rows.ctypes.data, M, arr, len(steps), int(f64),
                                            threads or os.cpu_count() or 1)
        if rc != 0:
            raise RuntimeError("oracle_fused_rows failed")
        out[bt * M:(bt + 1) * M] = part
    return out.reshape(*batch, M, N)


def add_oracle(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    oracle_lib().oracle_add(a.ctypes.data, a.size, b.ctypes.data, b.size, out.ctypes.data)
    return out


def relu_oracle(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    oracle_lib().oracle_relu(x.ctypes.data, x.size, out.ctypes.data)
    return out


# ------------------------------------------------------------------ reference host API


def ref_available() -> bool:
    return REF_LIB.exists()


def ref_lib():
    """The reference's tensor.c/graph.c/optimizer.c as a shared library."""
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError(f"{REF_LIB} missing: run `make -C oracle ref` where the reference sources exist")
        from minixla_b200.abi import EpStep, Node, Tensor

        lib = C.CDLL(str(REF_LIB))
        PT, PN = C.POINTER(Tensor), C.POINTER(Node)
        sig = {
            "create_tensor": (PT, [C.c_void_p, C.POINTER(C.c_int), C.c_int]),
            "free_tensor": (None, [PT]),
            "input_node": (PN, [PT]),
            "const_node": (PN, [PT]),
            "fused_node": (PN, [PN, PN, C.POINTER(EpStep), C.c_int]),
            "g_matmul": (PN, [PN, PN]),
            "g_add": (PN, [PN, PN]),
            "g_mul": (PN, [PN, PN]),
            "g_relu": (PN, [PN]),
            "g_transpose": (PN, [PN]),
            "optimize": (PN, [PN]),
            "execute": (PT, [PN]),
            "free_graph": (None, [PN]),
            "graph_collect": (C.c_int, [PN, C.POINTER(C.POINTER(PN))]),
            "matmul": (PT, [PT, PT]),
            "tensor_add": (PT, [PT, PT]),
            "relu": (PT, [PT]),
        }
        for name, (res, args) in sig.items():
            f = getattr(lib, name)
            f.restype, f.argtypes = res, args
        _ref = lib
    return _ref


class RefGraph:
    """Builds and evaluates graphs with the reference's own host API."""

    def __init__(self) -> None:
        self.lib = ref_lib()
        self._tensors = []
        self._roots = []

    def tensor(self, arr: np.ndarray):
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        shape = (C.c_int * arr.ndim)(*arr.shape)
        t = self.lib.create_tensor(arr.ctypes.data, shape, arr.ndim)  # copies the data
        if not t:
            raise RuntimeError("create_tensor failed")
        self._tensors.append(t)
        return t

    def input(self, arr: np.ndarray):
        return self.lib.input_node(self.tensor(arr))

    def const(self, arr: np.ndarray):
        return self.lib.const_node(self.tensor(arr))

    def fused(self, a, b, steps):
        from minixla_b200.abi import EpStep

        ep = (EpStep * max(1, len(steps)))(*[EpStep(op, operand) for op, operand in steps])
        return self.lib.fused_node(a, b, ep, len(steps))

    def optimize(self, root):
        return self.lib.optimize(root)

    def execute(self, root) -> np.ndarray:
        """The reference's CPU execute() (graph.c:131-149); memoizes into the graph."""
        t = self.lib.execute(root)
        if not t:
            raise RuntimeError("reference execute() failed")
        from minixla_b200.abi import tensor_to_numpy

        return tensor_to_numpy(t)

    def node_count(self, root) -> int:
        from minixla_b200.abi import Node

        out = C.POINTER(C.POINTER(Node))()
        n = self.lib.graph_collect(root, C.byref(out))
        C.CDLL(None).free(C.cast(out, C.c_void_p))
        return n

    def own(self, root):
        """Registers a root whose graph is freed by close()."""
        self._roots.append(root)
        return root

    def close(self) -> None:
        for r in self._roots:
            self.lib.free_graph(r)
        for t in self._tensors:
            self.lib.free_tensor(t)
        self._roots, self._tensors = [], []
