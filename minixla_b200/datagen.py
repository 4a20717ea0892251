"""Seeded, counter-based synthetic inputs for the fused relu(A.B+C) workloads.

Element i of stream s (one stream per tensor) comes from splitmix64's output
function applied to ``base(seed, s) + (i + 1) * GAMMA`` -- a counter-based
generator, so any row slice of a large matrix can be produced on its own and
matches the same rows of the full matrix.

* uniform[-1, 1): the top 24 bits u of the 64-bit draw, value = u * 2^-23 - 1
  (exact in fp32);
* normal(mu, sigma): Box-Muller in float64 from draws 2i and 2i+1, rounded to
  fp32 at the end.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_CHUNK = 1 << 21


def _mix(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * _M1
    z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def _base(seed: int, stream: int) -> np.uint64:
    with np.errstate(over="ignore"):
        x = np.array([(seed * 0x9E3779B97F4A7C15 + stream * 0xD1B54A32D192ED03 + 0x632BE59BD9B4E019)
                      % (1 << 64)], dtype=np.uint64)
        return _mix(x)[0]


def raw_bits(n: int, stream: int, seed: int = 0, offset: int = 0) -> np.ndarray:
    """n 64-bit draws of `stream` starting at counter `offset`."""
    base = _base(seed, stream)
    idx = np.arange(offset + 1, offset + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return _mix(base + idx * GAMMA)


def _chunked(n: int, fill) -> None:
    """Runs fill(c0, c1) over [0, n) in chunks; numpy releases the GIL, so
    chunks run on a small thread pool."""
    spans = [(c0, min(n, c0 + _CHUNK)) for c0 in range(0, n, _CHUNK)]
    if len(spans) <= 1:
        for c0, c1 in spans:
            fill(c0, c1)
        return
    with ThreadPoolExecutor(max_workers=min(len(spans), os.cpu_count() or 1, 16)) as ex:
        list(ex.map(lambda s: fill(*s), spans))


def uniform(shape, stream: int, seed: int = 0, row_offset: int = 0) -> np.ndarray:
    """float32 array of `shape`, i.i.d. uniform[-1, 1); rows start at `row_offset`."""
    shape = tuple(shape)
    cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    start = row_offset * cols

    def fill(c0, c1):
        u = (raw_bits(c1 - c0, stream, seed, start + c0) >> np.uint64(40)).astype(np.float32)
        out[c0:c1] = u * np.float32(2.0 ** -23) - np.float32(1.0)

    _chunked(n, fill)
    return out.reshape(shape)


def normal(shape, stream: int, mu: float = 0.0, sigma: float = 1.0, seed: int = 0,
           row_offset: int = 0) -> np.ndarray:
    """float32 array of `shape`, i.i.d. normal(mu, sigma); rows start at `row_offset`."""
    shape = tuple(shape)
    cols = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    start = row_offset * cols

    def fill(c0, c1):
        b = raw_bits(2 * (c1 - c0), stream, seed, 2 * (start + c0))
        u1 = ((b[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
        u2 = (b[1::2] >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
        z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
        out[c0:c1] = (mu + sigma * z).astype(np.float32)

    _chunked(n, fill)
    return out.reshape(shape)
