"""Regenerates tests/golden/golden.npz from MiniXLA's own CPU execute().

Runs where the reference host library has been built from the reference
sources (``make -C oracle ref``): every case in cases.py is built with the
reference's own constructors and evaluated by its execute() (graph.c:131-149,
eval_fused graph.c:64-115).  Outputs are stored with a SHA-256 of every
input (cases.py regenerates the inputs from the seeded generator, and the
digests pin that generator), so the tests can check the oracle and the GPU
path without the reference present.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from minixla_b200.abi import OP_ADD, OP_RELU  # noqa: E402
from oracle.bindings import RefGraph  # noqa: E402
from tests.golden.cases import all_cases  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden.npz"


def input_digest(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a, dtype=np.float32)
    return hashlib.sha256(repr(a.shape).encode() + a.tobytes()).hexdigest()


class RefBuilder:
    """cases.py builder interface over the reference's host API."""

    def __init__(self, rg: RefGraph):
        self.rg = rg

    def fused(self, a, b, steps):
        return self.rg.fused(a, b, [(OP_ADD if op == "add" else OP_RELU, n) for op, n in steps])

    def matmul(self, a, b):
        return self.rg.lib.g_matmul(a, b)

    def add(self, a, b):
        return self.rg.lib.g_add(a, b)

    def relu(self, x):
        return self.rg.lib.g_relu(x)


def main() -> None:
    arrays = {}
    for name, inputs, build in all_cases():
        rg = RefGraph()
        t = {k: rg.input(v) for k, v in inputs.items()}
        root = rg.own(build(RefBuilder(rg), t))
        out = rg.execute(root)
        rg.close()
        for k, v in inputs.items():
            arrays[f"{name}:{k}:sha256"] = np.array(input_digest(v))
        arrays[f"{name}:__out__"] = out
        print(f"{name}: out {out.shape}")
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
