"""Kernel choice per shape (mxb_gemm_plan_for), host-only: the rules the
dispatcher follows, on a 148-SM GPU, without a GPU.  The same plan function
drives the launches (launch_fused_gemm dispatches on it), so these cases pin
what the GPU runs."""
from pathlib import Path

import pytest

from minixla_b200 import lib as mlib

TF32, X3 = mlib.GPU_PRECISION_TF32, mlib.GPU_PRECISION_3XTF32
SKINNY, TINY, SINGLE, PAIR = (mlib.MXB_KERNEL_SKINNY, mlib.MXB_KERNEL_TINY, mlib.MXB_KERNEL_SINGLE_CTA,
                              mlib.MXB_KERNEL_CTA_PAIR)

# (M, N, K, precision) -> (kernel, tile_rows, tile_cols, k_splits)
CASES = [
    ((8192, 8192, 8192, TF32), (PAIR, 256, 512, 1)),      # headline: wide pair tiles
    ((8192, 8192, 8192, X3), (PAIR, 256, 256, 1)),
    ((32768, 8192, 8192, TF32), (PAIR, 256, 512, 1)),
    ((2048, 2048, 2048, TF32), (PAIR, 256, 256, 1)),      # too few 256 x 512 tiles
    ((4096, 8192, 4096, TF32), (PAIR, 256, 256, 1)),      # wide tiles would need a stream-K tail, K < 8192
    ((4096, 8192, 8192, TF32), (PAIR, 256, 512, 1)),      # ... at K = 8192 they keep it
    ((1024, 1024, 1024, TF32), (SINGLE, 128, 64, 1)),     # 32 k-blocks: no K split
    ((8191, 127, 3000, TF32), (SINGLE, 128, 128, 2)),     # few tiles, long K
    ((8191, 127, 3000, X3), (SINGLE, 128, 128, 2)),
    ((4096, 128, 2048, TF32), (SINGLE, 128, 128, 4)),
    ((760, 890, 4100, TF32), (SINGLE, 128, 128, 3)),     # 42 tiles: three slices per tile
    ((512, 512, 8192, TF32), (SINGLE, 128, 128, 8)),
    ((16, 8192, 8192, TF32), (SINGLE, 128, 128, 2)),      # 9..16 rows: tensor cores in TF32 mode
    ((9, 4096, 4096, TF32), (SINGLE, 128, 128, 4)),
    ((16, 8192, 8192, X3), (SKINNY, 16, 128, 8)),         # ... CUDA cores in 3xTF32 mode
    ((8, 8192, 8192, TF32), (SKINNY, 8, 128, 8)),
    ((1, 4096, 4096, TF32), (SKINNY, 1, 128, 8)),
    ((128, 128, 128, X3), (TINY, 32, 32, 1)),             # config 1 in 3xTF32 mode
    ((128, 128, 128, TF32), (SINGLE, 128, 32, 1)),
    ((257, 4097, 129, TF32), (SINGLE, 128, 128, 1)),     # 99 tiles of 128 x 128
    ((1, 4096, 4096, X3), (SKINNY, 1, 128, 8)),
]


@pytest.mark.parametrize("shape,want", CASES, ids=[f"{m}x{n}x{k}-{'tf32' if p == TF32 else '3x'}"
                                                   for (m, n, k, p), _ in CASES])
def test_plan(shape, want, monkeypatch):
    for var in ("MINIXLA_KSPLIT", "MINIXLA_SKINNY_MAX_ROWS", "MINIXLA_GEMM_VARIANT", "MINIXLA_SINGLE_BN",
                "MINIXLA_TINY_MAX_MNK", "MINIXLA_SKINNY_FORM"):
        monkeypatch.delenv(var, raising=False)
    p = mlib.gemm_plan(*shape)
    assert (p.kernel, p.tile_rows, p.tile_cols, p.k_splits) == want
    assert p.products == 1


def test_plan_follows_settings(monkeypatch):
    for var in ("MINIXLA_KSPLIT", "MINIXLA_SKINNY_MAX_ROWS", "MINIXLA_GEMM_VARIANT", "MINIXLA_SINGLE_BN"):
        monkeypatch.delenv(var, raising=False)
    monkeypatch.setenv("MINIXLA_KSPLIT", "0")
    p = mlib.gemm_plan(8191, 127, 3000, TF32)
    assert (p.kernel, p.tile_cols, p.k_splits) == (SINGLE, 64, 1)
    monkeypatch.setenv("MINIXLA_KSPLIT", "3")
    assert mlib.gemm_plan(8191, 127, 3000, TF32).k_splits == 3
    monkeypatch.delenv("MINIXLA_KSPLIT")
    monkeypatch.setenv("MINIXLA_SKINNY_MAX_ROWS", "16")
    assert mlib.gemm_plan(16, 8192, 8192, TF32).kernel == SKINNY
    monkeypatch.setenv("MINIXLA_SKINNY_MAX_ROWS", "0")
    assert mlib.gemm_plan(1, 4096, 4096, TF32).kernel == SINGLE
    assert mlib.gemm_plan(1, 4096, 4096, X3).kernel == TINY        # 2^24 <= 2^26 in 3xTF32 mode
    monkeypatch.delenv("MINIXLA_SKINNY_MAX_ROWS")
    monkeypatch.setenv("MINIXLA_GEMM_VARIANT", "single")
    p = mlib.gemm_plan(8192, 8192, 8192, TF32)
    assert (p.kernel, p.tile_cols) == (SINGLE, 256)
    monkeypatch.setenv("MINIXLA_GEMM_VARIANT", "pair")
    p = mlib.gemm_plan(8192, 8192, 8192, TF32)
    assert (p.kernel, p.tile_cols) == (PAIR, 256)
    monkeypatch.delenv("MINIXLA_GEMM_VARIANT")
    monkeypatch.setenv("MINIXLA_SINGLE_BN", "32")
    p = mlib.gemm_plan(8191, 127, 3000, TF32)
    assert (p.kernel, p.tile_cols, p.k_splits) == (SINGLE, 32, 1)   # a forced width runs unsplit


def test_plan_depends_on_sm_count():
    # Fewer SMs: the same 8192-row product already fills the GPU with 256 x 512 tiles.
    assert mlib.gemm_plan(2048, 2048, 2048, TF32, num_sms=32).tile_cols == 512
    # More tiles than half the SMs: no K split.
    assert mlib.gemm_plan(8191, 127, 3000, TF32, num_sms=100).k_splits == 1


@pytest.mark.parametrize("args", [(0, 8, 8, TF32, 148), (8, 8, 8, 2, 148), (8, 8, 8, TF32, 1)])
def test_plan_rejects_bad_arguments(args):
    with pytest.raises(ValueError):
        mlib.gemm_plan(*args)


# (batch, M, N, K, precision) -> (kernel, tile_rows, tile_cols, products per launch)
BATCH_CASES = [
    ((64, 256, 256, 256, TF32), (SINGLE, 128, 128, 64)),     # small products: one launch
    ((64, 256, 256, 256, X3), (SINGLE, 128, 128, 64)),
    ((16, 250, 130, 300, TF32), (SINGLE, 128, 128, 16)),
    ((5, 384, 520, 1000, TF32), (SINGLE, 128, 256, 5)),      # N >= 512: 128 x 256 tiles
    ((32, 1024, 1024, 1024, TF32), (PAIR, 256, 256, 32)),    # from 1024 x 1024: CTA pairs
    ((32, 1024, 1024, 1024, X3), (PAIR, 256, 256, 32)),
    ((3, 1100, 1030, 1056, X3), (PAIR, 256, 256, 3)),        # ragged, 75 pair tiles
    ((8, 1100, 1030, 300, X3), (SINGLE, 128, 128, 8)),       # short K: single-CTA tiles
    ((8, 2048, 2048, 2048, TF32), (PAIR, 256, 256, 1)),      # fills the GPU: one launch per product
    ((4, 8, 4096, 4096, TF32), (SKINNY, 8, 128, 1)),         # few rows: skinny kernel per product
    ((4, 64, 64, 64, X3), (TINY, 32, 32, 1)),                # tiny in total (3xTF32)
]


@pytest.mark.parametrize("shape,want", BATCH_CASES, ids=[f"{b}x{m}x{n}x{k}-{'tf32' if p == TF32 else '3x'}"
                                                         for (b, m, n, k, p), _ in BATCH_CASES])
def test_plan_batched(shape, want, monkeypatch):
    for var in ("MINIXLA_BATCH_LAUNCH", "MINIXLA_BATCH_PAIR", "MINIXLA_BATCH_WIDE", "MINIXLA_SKINNY_MAX_ROWS",
                "MINIXLA_TINY_MAX_MNK", "MINIXLA_GEMM_VARIANT"):
        monkeypatch.delenv(var, raising=False)
    b, m, n, k, prec = shape
    p = mlib.gemm_plan(m, n, k, prec, batch=b)
    assert (p.kernel, p.tile_rows, p.tile_cols, p.products) == want
    monkeypatch.setenv("MINIXLA_BATCH_LAUNCH", "0")
    assert mlib.gemm_plan(m, n, k, prec, batch=b).products == 1



# (M, N, K) -> stream-K tiles on 74 CTA pairs (TF32): tiles that do not make a
# whole last wave are shared out by k-blocks over every pair.
STREAMK = [
    ((4096, 4096, 4096), 0),      # 128 tiles: fewer than two whole waves, all in step instead
    ((4096, 8192, 8192), 108),    # the 8-way split of 32768 x 8192 x 8192: 256 tiles = 3 x 74 + 34
    ((6144, 8192, 8192), 88),     # 384 tiles = 5 x 74 + 14: 60 idle pair-tiles; the last 88 stream-K
    ((8192, 8192, 8192), 0),      # 512 tiles = 6 x 74 + 68: 6 idle pair-tiles, under 1 in 25
    ((32768, 8192, 8192), 0),     # 2048 tiles = 27 x 74 + 50: 24 idle, under 1 in 25
    ((2048, 2048, 2048), 0),      # 64 tiles of 256 x 256: fewer than the pairs
    ((9472, 8192, 8192), 0),      # 592 tiles = 8 x 74 exactly
    ((5120, 4096, 2048), 98),     # 256 x 256 tiles (see below): 320 = 4 x 74 + 24
    ((5120, 4096, 1024), 0),      # ... with a short k-loop (32 blocks)
    ((3300, 6001, 2049), 90),     # 312 tiles of 256 x 256 = 4 x 74 + 16, ragged M, N, K
]


@pytest.mark.parametrize("shape,want", STREAMK, ids=[f"{m}x{n}x{k}" for (m, n, k), _ in STREAMK])
def test_streamk_tiles(shape, want, monkeypatch):
    for var in ("MINIXLA_STREAMK", "MINIXLA_GEMM_VARIANT"):
        monkeypatch.delenv(var, raising=False)
    assert mlib.gemm_plan(*shape, TF32).streamk_tiles == want
    assert mlib.gemm_plan(*shape, X3).streamk_tiles == 0   # 3xTF32 pair kernel: whole tiles
    monkeypatch.setenv("MINIXLA_STREAMK", "0")
    assert mlib.gemm_plan(*shape, TF32).streamk_tiles == 0


def test_streamk_schedule_covers_every_kblock_once(tmp_path):
    """The stream-K work lists themselves (pair_work / streamk_split from
    gemm_common.cuh, compiled for the host): every k-block of every tile runs
    on exactly one pair; a split tile is shared by two neighbouring pairs, as
    the first item of one and the last of the next (the accumulator hand-off
    the kernel implements), coming after the pair's whole-wave tiles and last
    on the next pair's list; the pairs' stream-K k-blocks differ by at most one."""
    import random
    import shutil
    import subprocess

    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    root = Path(__file__).resolve().parents[1]
    exe = tmp_path / "streamk_schedule"
    subprocess.run([nvcc, "-std=c++17", "-O1", "-gencode", "arch=compute_100a,code=sm_100a", "-I",
                    str(root / "include"), "--expt-relaxed-constexpr", "-o", str(exe),
                    str(root / "tests" / "native" / "streamk_schedule.cu"),
                    str(root / "minixla_b200" / "csrc" / "tensor_maps.cu")], check=True, capture_output=True)
    rng = random.Random(7)
    cases = [(128, 128, 74), (512, 256, 74), (256, 256, 74), (2048, 256, 74), (75, 1, 74), (149, 3, 74),
             (64, 64, 74), (74, 9, 74), (1000, 33, 73), (3, 5, 2)]
    cases += [(rng.randint(1, 3000), rng.randint(1, 300), rng.randint(2, 80)) for _ in range(300)]
    out = subprocess.run([str(exe)] + [str(x) for c in cases for x in c], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == f"OK {len(cases)}", out.stdout
