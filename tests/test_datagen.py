"""CPU tests of the seeded input generator."""
import numpy as np

from minixla_b200 import datagen


def test_uniform_is_deterministic_and_in_range():
    a = datagen.uniform((64, 33), stream=3)
    b = datagen.uniform((64, 33), stream=3)
    assert np.array_equal(a, b)
    assert a.dtype == np.float32 and a.min() >= -1.0 and a.max() < 1.0
    assert abs(float(a.mean())) < 0.05
    # Values sit on the 2^-23 grid (24 random bits).
    assert np.all((a.astype(np.float64) + 1.0) * 2**23 == np.round((a.astype(np.float64) + 1.0) * 2**23))


def test_streams_differ():
    assert not np.array_equal(datagen.uniform((100,), 0), datagen.uniform((100,), 1))


def test_row_slices_match_full_matrix():
    full = datagen.uniform((50, 17), stream=5)
    part = datagen.uniform((10, 17), stream=5, row_offset=20)
    assert np.array_equal(part, full[20:30])
    fulln = datagen.normal((40, 9), stream=6, mu=0.5, sigma=2.0)
    partn = datagen.normal((5, 9), stream=6, mu=0.5, sigma=2.0, row_offset=33)
    assert np.array_equal(partn, fulln[33:38])


def test_normal_moments():
    x = datagen.normal((200000,), stream=7, mu=1.0, sigma=0.5).astype(np.float64)
    assert abs(x.mean() - 1.0) < 0.01 and abs(x.std() - 0.5) < 0.01


def test_chunk_boundaries_are_seamless():
    n = (1 << 21) * 2 + 10
    x = datagen.uniform((n,), stream=9)
    y = datagen.uniform((20,), stream=9, row_offset=(1 << 21) - 10)
    assert np.array_equal(x[(1 << 21) - 10:(1 << 21) + 10], y)
