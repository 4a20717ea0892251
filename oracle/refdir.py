"""Where the reference sources are, for the recipes that compile the CPU
checkers and the drop-in test programs -- TEST INFRASTRUCTURE ONLY.

$MINIXLA_REF_DIR when set, else ``baseline/_ref`` when it holds the sources,
else the read-only checkout the recipes were written against.  None when no
candidate has the sources (the GPU box, for one: there the prebuilt
``oracle/_ref`` files are used instead)."""
from __future__ import annotations

import os
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
_CHECKOUT = Path("/root/reference")


def ref_dir() -> Path | None:
    env = os.environ.get("MINIXLA_REF_DIR")
    candidates = [Path(env)] if env else [ROOT / "baseline" / "_ref", _CHECKOUT]
    for c in candidates:
        if (c / "graph.c").exists():
            return c
    return None
