"""Row all-gather fused into the GEMM epilogue (mxb_fused_gemm_allgather with
minixla_b200.peer_gather.GatherBuffers), one process per GPU.

CPU (gloo, world size 2): the host-side plumbing against a fake library --
handle exchange, peer addresses in rank order, the arguments of the launch,
unmap-before-free on close.

GPU (one process per visible GPU, up to eight, NCCL): every rank's full buffer after the
fused gather must equal, bit for bit, the NCCL all-gather of the same
shards computed by mxb_fused_gemm, and sampled rows must match the oracle.
Covers the in-kernel push (TF32 256 x 256 and 256 x 512 pair tiles, the
3xTF32 pair kernel, float4 and odd-pitch scalar copies, uneven shards) and
the copy form (the single-CTA and skinny kernels, MINIXLA_GATHER_PUSH=0)."""
import ctypes as C
import os
import socket
from datetime import timedelta

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


# ---------------------------------------------------------------- CPU: host plumbing with a fake library


class _FakeLib:
    """Stands in for the native library: buffer addresses encode the owning
    rank, handles carry the address, mappings add a per-process offset."""

    MAP_BASE = 0x7F0000000000

    def __init__(self, rank):
        self.rank = rank
        self.calls = []

    def mxb_ipc_alloc(self, device, nbytes, ptr_ref, handle):
        addr = 0x100000000 * (self.rank + 1)
        ptr_ref._obj.value = addr
        raw = addr.to_bytes(8, "little") + nbytes.to_bytes(8, "little")
        for i, b in enumerate(raw):
            handle[i] = b
        self.calls.append(("alloc", device, nbytes))
        return 0

    def mxb_ipc_open(self, device, handle, ptr_ref):
        addr = int.from_bytes(bytes(handle[:8]), "little")
        ptr_ref._obj.value = self.MAP_BASE + addr
        self.calls.append(("open", device, addr))
        return 0

    def mxb_ipc_close(self, device, ptr):
        self.calls.append(("close", device, ptr))
        return 0

    def mxb_ipc_free(self, device, ptr):
        self.calls.append(("free", device, ptr))
        return 0

    def mxb_fused_gemm_allgather(self, ctx, A, lda, B, ldb, out, ldo, peers, n, M, N, K, steps, n_steps, prec, st):
        self.calls.append(("gemm", out, ldo, [peers[i] for i in range(n)], n, M, N, K))
        return 0


def _cpu_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        import sys
        sys.path.insert(0, os.getcwd())
        from minixla_b200.peer_gather import GatherBuffers

        lib = _FakeLib(rank)
        rows, cols, ldo = 1000, 60, 64
        gb = GatherBuffers(lib, device=rank, rows_total=rows, cols=cols, ldo=ldo)
        row0 = 500 * rank
        gb.gemm(ctx=None, A=1, lda=4, B=2, ldb=64, row0=row0, M=500, N=cols, K=4, steps=None, n_steps=0,
                precision=1, stream=0)
        gb.close()
        q.put((rank, lib.calls))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


def test_gather_buffers_host_logic_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_cpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        calls = out[rank]
        assert isinstance(calls, list), calls
        nbytes = 4 * 1000 * 64
        assert calls[0] == ("alloc", rank, nbytes)
        peer = 1 - rank
        peer_addr = 0x100000000 * (peer + 1)
        own_addr = 0x100000000 * (rank + 1)
        assert calls[1] == ("open", rank, peer_addr)
        kind, out_ptr, ldo, peers, n, M, N, K = calls[2]
        row0 = 500 * rank
        assert kind == "gemm" and ldo == 64 and n == 1 and (M, N, K) == (500, 60, 4)
        assert out_ptr == own_addr + 4 * row0 * 64
        assert peers == [_FakeLib.MAP_BASE + peer_addr + 4 * row0 * 64]
        # the peer's mapping is closed before this rank frees its own buffer
        assert calls[3] == ("close", rank, _FakeLib.MAP_BASE + peer_addr)
        assert calls[4] == ("free", rank, own_addr)


def _cpu_checks_worker(port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=timedelta(seconds=60))
        import sys
        sys.path.insert(0, os.getcwd())
        from minixla_b200.peer_gather import GatherBuffers

        errors = []
        try:
            GatherBuffers(_FakeLib(0), device=0, rows_total=10, cols=8, ldo=4)
        except ValueError as e:
            errors.append(("ldo", str(e)))
        lib = _FakeLib(0)
        gb = GatherBuffers(lib, device=0, rows_total=100, cols=8)
        for row0, M, N in ((-1, 10, 8), (95, 10, 8), (0, 10, 9)):
            try:
                gb.gemm(None, 1, 4, 2, 8, row0, M, N, 4, None, 0, 1, 0)
            except ValueError as e:
                errors.append(("rows", str(e)))
        ptrs, n = gb.peer_rows(7)
        launched = [c for c in lib.calls if c[0] == "gemm"]
        gb.close()
        gb.close()  # a second close is a no-op
        q.put((errors, n, len(launched), [c[0] for c in lib.calls]))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put(repr(e))


def test_gather_buffers_argument_checks():
    """One rank (gloo): a pitch narrower than the rows, rows outside the
    buffer and a column count other than the buffer's are refused before any
    launch; with no peers the launch gets an empty peer list; close is
    idempotent and frees the buffer once."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_cpu_checks_worker, args=(port, q))
    p.start()
    res = q.get(timeout=120)
    p.join(timeout=60)
    assert p.exitcode == 0
    assert isinstance(res, tuple), res
    errors, n_peers, launched, calls = res
    assert [k for k, _ in errors] == ["ldo", "rows", "rows", "rows"]
    assert n_peers == 0 and launched == 0
    assert calls == ["alloc", "free"]


# ---------------------------------------------------------------- GPU: one process per GPU

# (rows per rank, extra rows, N, K, precision, MINIXLA_GATHER_PUSH, expect the
# in-kernel push): M = rows per rank x ranks + extra, so every rank runs the
# same kernel family whatever the GPU count.
GPU_CASES = [
    (2048, 0, 2048, 256, 1, "1", True),    # 256 x 256 pair tiles, TMA tile stores
    (4096, 0, 4096, 128, 1, "1", True),    # 256 x 512 pair tiles
    (4096, 0, 6144, 2048, 1, "1", True),   # 384 tiles of 256 x 256 per shard: stream-K tail (88) with the push
    (2048, 1, 2047, 200, 1, "1", True),    # uneven shards, odd pitch: scalar copies, K tail
    (2048, 0, 2048, 256, 1, "0", False),   # copy form forced
    (2048, 0, 2048, 256, 3, "1", True),    # 3xTF32 CTA-pair kernel pushes too
    (2048, 1, 2047, 200, 3, "1", True),    # ... with uneven shards and an odd pitch
    (100, 0, 96, 64, 1, "1", False),       # single-CTA kernel
    (8, 0, 512, 256, 1, "1", False),       # skinny kernel
]


def _gpu_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
        import sys
        sys.path.insert(0, os.getcwd())
        from minixla_b200 import datagen
        from minixla_b200 import lib as mlib
        from minixla_b200.peer_gather import GatherBuffers
        from oracle.bindings import fused_oracle

        lib = mlib.load()
        ctx = lib.gpu_ctx_create_on(rank)
        assert ctx, mlib.last_error()
        stream = torch.cuda.Stream(dev)
        results = []
        for (per_rank, extra, N, K, prec, push_env, _) in GPU_CASES:
            M = per_rank * world + extra
            os.environ["MINIXLA_GATHER_PUSH"] = push_env
            r0, r1 = C.c_longlong(), C.c_longlong()
            assert lib.mxb_shard_rows(M, world, rank, C.byref(r0), C.byref(r1)) == 0
            r0, r1 = r0.value, r1.value
            A = datagen.uniform((M, K), 40)
            B = datagen.uniform((K, N), 41)
            Cm = datagen.normal((M, N), 42)
            ldb = (N + 3) // 4 * 4
            Bp = np.zeros((K, ldb), np.float32)
            Bp[:, :N] = B
            A_d = torch.from_numpy(np.ascontiguousarray(A[r0:r1])).to(dev)
            B_d = torch.from_numpy(Bp).to(dev)
            C_d = torch.from_numpy(np.ascontiguousarray(Cm[r0:r1])).to(dev)
            steps = (mlib.EpStepDev * 2)()
            steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, C_d.data_ptr(), N, 0.0, 0)
            steps[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
            gb = GatherBuffers(lib, rank, M, N, ldo=N)
            torch.cuda.synchronize()
            before = lib.mxb_gather_push_count()
            rc = gb.gemm(ctx, A_d.data_ptr(), K, B_d.data_ptr(), ldb, r0, r1 - r0, N, K, steps, 2, prec,
                         stream.cuda_stream)
            assert rc == 0, mlib.last_error()
            pushed = lib.mxb_gather_push_count() - before
            gb.barrier(stream)
            stream.synchronize()
            full = gb.tensor().clone()
            # the same shards through mxb_fused_gemm, gathered with NCCL
            ref = torch.empty((r1 - r0, N), device=dev)
            with torch.cuda.stream(stream):
                assert lib.mxb_fused_gemm(ctx, A_d.data_ptr(), K, B_d.data_ptr(), ldb, ref.data_ptr(), N, r1 - r0, N,
                                          K, steps, 2, prec, stream.cuda_stream) == 0, mlib.last_error()
            stream.synchronize()
            rows_max = (M + world - 1) // world
            padded = torch.zeros((rows_max, N), device=dev)
            padded[: r1 - r0] = ref
            parts = [torch.empty_like(padded) for _ in range(world)]
            dist.all_gather(parts, padded)
            bounds = []
            for r in range(world):
                a, b = C.c_longlong(), C.c_longlong()
                lib.mxb_shard_rows(M, world, r, C.byref(a), C.byref(b))
                bounds.append((a.value, b.value))
            ref_full = torch.cat([parts[r][: b - a] for r, (a, b) in enumerate(bounds)])
            exact = bool(torch.equal(full, ref_full))
            # sampled rows against the oracle: shard edges and a few inside
            rows = sorted({0, M - 1, *[x for a, b in bounds for x in (a, b - 1, (a + b) // 2)]})
            got = full[rows].cpu().numpy()
            want = fused_oracle(A[rows], B, [("add", Cm[rows]), ("relu",)])
            err = float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))
            results.append({"case": (M, N, K, prec, push_env), "pushed": int(pushed), "exact": exact, "err": err})
            gb.close()
            del A_d, B_d, C_d, ref, padded, parts, full, ref_full
        lib.gpu_ctx_destroy(ctx)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, results))
    except Exception as e:  # reported to the parent
        import traceback
        q.put((rank, traceback.format_exc() + repr(e)))


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.gpu
@pytest.mark.skipif(_ngpu() < 2, reason="needs at least two GPUs")
def test_fused_allgather_all_gpus():
    world, port = min(_ngpu(), 8), _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=600) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.exitcode is None:
                p.terminate()
    for rank in range(world):
        res = out[rank]
        assert isinstance(res, list), res
        for r, (_, _, N, K, prec, push_env, expect_push) in zip(res, GPU_CASES):
            assert r["exact"], r
            assert r["err"] <= (2e-3 if prec == 1 else 1e-5), r
            assert r["pushed"] == (1 if expect_push else 0), r
    for p in procs:
        assert p.exitcode == 0


def test_peer_order_starts_after_this_rank():
    """Every rank lists its peers starting with the next rank, so at any
    moment the ranks' first stores go to different GPUs (host-only)."""
    from minixla_b200.peer_gather import GatherBuffers

    for world in (2, 4, 8):
        firsts = []
        for rank in range(world):
            gb = GatherBuffers.__new__(GatherBuffers)
            gb.rank, gb.world = rank, world
            order = gb.peer_order()
            assert sorted(order) == [r for r in range(world) if r != rank]
            assert order == [(rank + i) % world for i in range(1, world)]
            firsts.append(order[0])
        assert sorted(firsts) == list(range(world))
