"""World-size-2 gloo tests on CPU of the row-sharding logic the multi-GPU
paths use: the library's row split (mxb_shard_rows), per-rank evaluation of
a row shard, the all-gather that rebuilds an intermediate read whole by a
later node, and the max-over-ranks timing reduction bench.py uses.  The CPU
oracle stands in for each GPU's kernel and gloo for NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard(lib, M, parts, part):
    import ctypes as C

    r0, r1 = C.c_longlong(), C.c_longlong()
    assert lib.mxb_shard_rows(M, parts, part, C.byref(r0), C.byref(r1)) == 0
    return r0.value, r1.value


def _worker(rank, world, port, M, K, N, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import sys
        sys.path.insert(0, os.getcwd())
        from minixla_b200 import datagen, lib as mlib
        from oracle.bindings import fused_oracle

        lib = mlib.load()
        X = datagen.uniform((M, K), 80)
        W = datagen.normal((K, K), 81, 0.0, 1.0 / np.sqrt(K))
        b = datagen.normal((K,), 82, 0.0, 0.1)
        V = datagen.normal((M, K), 83)
        r0, r1 = _shard(lib, M, world, rank)
        # layer 1 on this rank's rows: H = relu(X W + b), rows [r0, r1)
        H_shard = fused_oracle(X[r0:r1], W, [("add", b), ("relu",)])
        # a later node reads H whole (as its B operand): all-gather the uneven shards
        counts = [_shard(lib, M, world, r)[1] - _shard(lib, M, world, r)[0] for r in range(world)]
        padded = torch.zeros((max(counts), K))
        padded[: r1 - r0] = torch.from_numpy(H_shard)
        gathered = [torch.zeros_like(padded) for _ in range(world)]
        dist.all_gather(gathered, padded)
        H = np.concatenate([g[:c].numpy() for g, c in zip(gathered, counts)])
        # layer 2, row-sharded again: out = X H[:K] + V, reading the gathered H whole as its B operand
        out_shard = fused_oracle(X[r0:r1], H[:K], [("add", V[r0:r1])])
        shards = [None] * world
        dist.all_gather_object(shards, (r0, r1, out_shard))
        # max-over-ranks, as bench.py reduces device times
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full_H = fused_oracle(X, W, [("add", b), ("relu",)])
            full_out = fused_oracle(X, full_H[:K], [("add", V)])
            rows = np.concatenate([np.arange(s[0], s[1]) for s in shards])
            out = np.concatenate([s[2] for s in shards])
            q.put(("ok", bool(np.array_equal(rows, np.arange(M))), bool(np.array_equal(H, full_H)),
                   bool(np.array_equal(out, full_out)), float(t.item())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("error", repr(e)))


@pytest.mark.parametrize("M", [64, 67])
def test_row_shards_rebuild_full_result_world2(M):
    world, K, N = 2, 48, 40
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, K, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
    assert res[0] == "ok", res
    _, covers, h_ok, out_ok, tmax = res
    assert covers and h_ok and out_ok
    assert tmax == float(world)


def test_shard_rows_partition():
    from minixla_b200 import lib as mlib

    lib = mlib.load()
    for M, parts in [(0, 3), (1, 8), (7, 8), (32768, 8), (1001, 4), (10, 1)]:
        spans = [_shard(lib, M, parts, p) for p in range(parts)]
        assert spans[0][0] == 0 and spans[-1][1] == M
        assert all(spans[i][1] == spans[i + 1][0] for i in range(parts - 1))
        sizes = [b - a for a, b in spans]
        assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_bench_strong_split_and_checked_rows(world):
    """bench.py's `strong` leg (config 5, 32768 x 8192 x 8192 split over N
    GPUs): its row split is the library's (mxb_shard_rows), the shards cover
    the job exactly once, and the rows each rank checks against the oracle
    are at least 64, inside the shard, and include both shard edges and both
    sides of the job's first 256-row tile boundary inside the shard (further
    boundaries are taken at a stride that keeps about eight of them)."""
    import bench
    from minixla_b200 import lib as mlib

    lib = mlib.load()
    covered = 0
    for rank in range(world):
        r0, r1, m_total = bench.shard_rows(world, rank, "strong")
        assert m_total == 32768 and (r0, r1) == _shard(lib, m_total, world, rank)
        covered += r1 - r0
        M = r1 - r0
        rows = bench.check_rows(M, r0)
        assert len(rows) >= 64 and rows == sorted(set(rows)) and 0 <= rows[0] and rows[-1] < M
        assert {0, 1, M - 2, M - 1} <= set(rows)
        # the first tile boundary of the job inside the shard, both sides
        first = (r0 + 255) // 256 * 256
        if r0 < first < r1:
            assert {first - r0 - 1, first - r0} <= set(rows)
    assert covered == 32768
