"""ctypes mirror of MiniXLA's host data model and the graph constructors the
hot path needs.

The layouts restate tensor.h:6-12 (``Tensor``) and graph.h:6-31 (``OpType``,
``EpStep``, ``Node``) of gouthamk16/miniXLA byte for byte; the C library reads
these structs in place.  The constructors mirror graph.c:20-59 for the nodes
``optimize()`` leaves behind on the hot path:

* ``input_node``  -- graph.c:20-24, an OP_INPUT leaf over a caller-owned tensor;
* ``fused_node``  -- graph.c:32-52, ``inputs = [a, b, ADD operands in step order]``;
* ``g_matmul`` / ``g_add`` / ``g_relu`` -- graph.c:54-57.

Host tensors here wrap numpy arrays (or torch CPU tensors, e.g. pinned ones)
without copying; a ``HostGraph`` keeps every buffer and struct alive for as
long as the graph is in use.
"""
from __future__ import annotations

import ctypes as C
from typing import Iterable, Sequence

import numpy as np

OP_INPUT, OP_MATMUL, OP_ADD, OP_MUL, OP_RELU, OP_SOFTMAX, OP_TRANSPOSE, OP_FUSED = range(8)


class Tensor(C.Structure):
    _fields_ = [
        ("data", C.POINTER(C.c_float)),
        ("shape", C.POINTER(C.c_int)),
        ("strides", C.POINTER(C.c_size_t)),
        ("ndim", C.c_int),
        ("size", C.c_size_t),
    ]


class Node(C.Structure):
    pass


class EpStep(C.Structure):
    _fields_ = [("op", C.c_int), ("operand", C.POINTER(Node))]


Node._fields_ = [
    ("op", C.c_int),
    ("inputs", C.POINTER(C.POINTER(Node))),
    ("n_inputs", C.c_int),
    ("output", C.POINTER(Tensor)),
    ("owns_output", C.c_int),
    ("visited", C.c_char),
    ("uses", C.c_int),
    ("is_const", C.c_char),
    ("epilogue", C.POINTER(EpStep)),
    ("n_epilogue", C.c_int),
]

assert C.sizeof(Tensor) == 40 and C.sizeof(EpStep) == 16 and C.sizeof(Node) == 64


class HostGraph:
    """Owns the structs and host buffers of one graph built from Python."""

    def __init__(self) -> None:
        self._keep: list = []

    # -- tensors --------------------------------------------------------
    def tensor(self, data) -> C.POINTER(Tensor):
        """Wraps a C-contiguous float32 numpy array or CPU torch tensor (no copy)."""
        if isinstance(data, np.ndarray):
            if data.dtype != np.float32 or not data.flags["C_CONTIGUOUS"]:
                raise ValueError("host tensors must be C-contiguous float32")
            ptr, shape = data.ctypes.data, data.shape
        else:  # torch.Tensor
            if str(data.dtype) != "torch.float32" or not data.is_contiguous() or data.device.type != "cpu":
                raise ValueError("host tensors must be contiguous float32 CPU tensors")
            ptr, shape = data.data_ptr(), tuple(data.shape)
        if len(shape) == 0 or any(s <= 0 for s in shape):
            raise ValueError("every dimension must be positive (create_tensor, tensor.c:8-24)")
        nd = len(shape)
        shp = (C.c_int * nd)(*shape)
        strides, acc = [0] * nd, 1
        for i in range(nd - 1, -1, -1):
            strides[i] = acc
            acc *= shape[i]
        strd = (C.c_size_t * nd)(*strides)
        t = Tensor(C.cast(C.c_void_p(ptr), C.POINTER(C.c_float)), shp, strd, nd, acc)
        self._keep += [data, shp, strd, t]
        return C.pointer(t)

    # -- nodes ----------------------------------------------------------
    def _node(self, op: int, inputs: Sequence) -> C.POINTER(Node):
        n = Node()
        n.op = op
        n.n_inputs = len(inputs)
        if inputs:
            arr = (C.POINTER(Node) * len(inputs))(*inputs)
            n.inputs = C.cast(arr, C.POINTER(C.POINTER(Node)))
            self._keep.append(arr)
        self._keep.append(n)
        return C.pointer(n)

    def input_node(self, data) -> C.POINTER(Node):
        p = self._node(OP_INPUT, [])
        p.contents.output = self.tensor(data)
        return p

    def fused_node(self, a, b, steps: Iterable[tuple[int, object]]) -> C.POINTER(Node):
        """steps: (OP_ADD, operand_node) or (OP_RELU, None), in order."""
        steps = list(steps)
        adds = [operand for op, operand in steps if op == OP_ADD]
        p = self._node(OP_FUSED, [a, b, *adds])
        if steps:
            ep = (EpStep * len(steps))(*[EpStep(op, operand if operand is not None else None) for op, operand in steps])
            p.contents.epilogue = C.cast(ep, C.POINTER(EpStep))
            p.contents.n_epilogue = len(steps)
            self._keep.append(ep)
        return p

    def g_matmul(self, a, b):
        return self._node(OP_MATMUL, [a, b])

    def g_add(self, a, b):
        return self._node(OP_ADD, [a, b])

    def g_relu(self, x):
        return self._node(OP_RELU, [x])


def tensor_to_numpy(t: C.POINTER(Tensor)) -> np.ndarray:
    """Copies a library-returned host tensor into a new numpy array."""
    shape = tuple(t.contents.shape[i] for i in range(t.contents.ndim))
    n = int(t.contents.size)
    buf = np.ctypeslib.as_array(t.contents.data, shape=(n,)).copy()
    return buf.reshape(shape)


_libc = C.CDLL(None)
_libc.free.argtypes = [C.c_void_p]


def free_host_tensor(t: C.POINTER(Tensor)) -> None:
    """Releases a tensor the library returned, as the reference's free_tensor does (tensor.c:297-303)."""
    if not t:
        return
    _libc.free(C.cast(t.contents.data, C.c_void_p))
    _libc.free(C.cast(t.contents.shape, C.c_void_p))
    _libc.free(C.cast(t.contents.strides, C.c_void_p))
    _libc.free(C.cast(t, C.c_void_p))
