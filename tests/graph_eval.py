"""Evaluates a cases.py graph on the CPU oracle, and runs it on the GPU library.

``OracleBuilder`` computes each node eagerly with the C restatement of
eval_fused / tensor_add / relu (oracle/fused_oracle.c), giving the same
values as MiniXLA's execute() bit for bit.  ``HostBuilder`` builds the same
graph as ctypes Node structs for gpu_execute.
"""
from __future__ import annotations

import numpy as np

from minixla_b200.abi import OP_ADD, OP_RELU, HostGraph
from oracle.bindings import add_oracle, fused_oracle, fused_oracle_batched, relu_oracle


class OracleBuilder:
    def fused(self, a, b, steps):
        st = [("add", op) if kind == "add" else ("relu",) for kind, op in steps]
        return fused_oracle(a, b, st) if a.ndim == 2 else fused_oracle_batched(a, b, st)

    def matmul(self, a, b):
        return fused_oracle(a, b, []) if a.ndim == 2 else fused_oracle_batched(a, b, [])

    def add(self, a, b):
        return add_oracle(a, b)

    def relu(self, x):
        return relu_oracle(x)


def oracle_eval(inputs, build):
    return build(OracleBuilder(), dict(inputs))


class HostBuilder:
    def __init__(self, hg: HostGraph):
        self.hg = hg

    def fused(self, a, b, steps):
        return self.hg.fused_node(a, b, [(OP_ADD if k == "add" else OP_RELU, n) for k, n in steps])

    def matmul(self, a, b):
        return self.hg.g_matmul(a, b)

    def add(self, a, b):
        return self.hg.g_add(a, b)

    def relu(self, x):
        return self.hg.g_relu(x)


def host_graph(inputs, build):
    hg = HostGraph()
    t = {k: hg.input_node(np.ascontiguousarray(v, dtype=np.float32)) for k, v in inputs.items()}
    root = build(HostBuilder(hg), t)
    return hg, root


def rel_frobenius(got: np.ndarray, want: np.ndarray) -> float:
    got = got.astype(np.float64)
    want = want.astype(np.float64)
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))
