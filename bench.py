#!/usr/bin/env python
"""Benchmark of the fused relu(A.B + C) hot path (MiniXLA's OP_FUSED node) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one fused relu(A.B + C) over one batch of rows, fp32 in and out.
Workload of `value`: every GPU owns an 8192-row shard of A and C with the
full 8192 x 8192 B (weak scaling: the single-GPU case is the 8192^3 headline
shape).  Output rows stay on their GPU; no collective runs on the data path.
`--workload strong` makes `value` the fixed 32768 x 8192 x 8192 job instead.

ours:      `value` = whole-job TFLOP/s with inputs resident in HBM, K launches of
           the fused kernel through the device-pointer C ABI, timed with CUDA
           events on the launch stream, max over ranks.
           `e2e` = the same metric through gpu_execute() -- the reference's own
           entry point -- on pageable (malloc'd) host buffers, the returned
           tensor freed inside the step; `e2e.pinned_into` is the additive
           gpu_execute_into() with pinned buffers.
           `precision_3xtf32` = the default (fp32-faithful) mode, same loop.
           `strong` = the fixed 32768 x 8192 x 8192 job split by rows over the
           N GPUs: kernel only, with the row all-gather fused into the
           epilogue and with an NCCL all-gather after the kernel; speed-up and
           efficiency against the whole job on one GPU of the same run; >= 64
           rows per rank checked against the oracle.
           `sharded_executor` (N > 1) = the same job through the product's
           one-process multi-GPU executor (gpu_ctx_create_multi + gpu_execute).
           `allgather` = the all-gathers on the 8192-row shards of `value`.
reference: MiniXLA's own CPU execute() (eval_fused, graph.c:64-115), compiled
           unmodified from the reference sources into oracle/_ref, on a bounded
           row sample of the same workload using all host cores (one process per
           core, row-parallel), rank 0 only.  The reference has no multi-GPU
           path, so its value does not depend on N.
"""
from __future__ import annotations

import argparse
import ctypes as C
import datetime as dt
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

NDIM = 8192       # N = K = 8192
ROWS_PER_GPU = 8192
STRONG_M = 32768


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--precision", choices=["tf32", "3xtf32"], default="tf32")
    # "config5" is the earlier name of "strong", still accepted.
    p.add_argument("--workload", choices=["weak", "strong", "config5"], default="weak")
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    p.add_argument("--no-strong", action="store_true",
                   help="skip the 32768 x 8192 x 8192 strong-scaling and multi-GPU executor legs")
    p.add_argument("--sweep", action="store_true",
                   help="time every benchmark shape (kernel only, operands resident); one JSON line per shape")
    p.add_argument("--kernels", action="store_true",
                   help="HBM-bound kernels alone (standalone add / relu, skinny GEMM) on operands larger than L2: "
                        "GB/s against the measured copy rate; one JSON line per kernel")
    p.add_argument("--mlp", action="store_true",
                   help="the 3-layer MLP (X 4096 x 1024, hidden 4096) end to end, built with the reference's g_* API "
                        "and optimize(), "
                        "run through gpu_execute_into, weights uploaded or kept resident; one JSON line per run")
    p.add_argument("--shape", type=int, default=0,
                   help="per-GPU M = N = K override (profiling on a smaller case); 0 = 8192")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--batched", default="",
                   help="time a rank-3 fused node relu(A.B + C) of 'B,M,N,K' through gpu_time_kernel_ms, both modes, "
                        "one launch for the batch and one launch per product (one JSON line each)")
    p.add_argument("--mnk", default="",
                   help="with --sweep: time only this product, 'M,N,K' (no MLP; for profiling one kernel)")
    return p.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def shard_rows(world: int, rank: int, workload: str, rows_per_gpu: int = 0):
    """Row range [r0, r1) of this rank and the job's total M."""
    if rows_per_gpu:
        return rank * rows_per_gpu, (rank + 1) * rows_per_gpu, rows_per_gpu * world
    if workload in ("strong", "config5"):
        m_total = STRONG_M
        base, extra = divmod(m_total, world)
        r0 = rank * base + min(rank, extra)
        return r0, r0 + base + (1 if rank < extra else 0), m_total
    return rank * ROWS_PER_GPU, (rank + 1) * ROWS_PER_GPU, ROWS_PER_GPU * world


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, physical_index: str):
        self.idx = physical_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", self.idx], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.5)

    def stop(self, t0: float, t1: float):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = []
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                ts = dt.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        inside = [r for r in rows if t0 <= r[0] <= t1] or sorted(rows, key=lambda r: abs(r[0] - (t0 + t1) / 2))[:3]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[3]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in inside) if inside else None,
                "sm_max_mhz": max(r[2] for r in inside) if inside else None,
                "reasons": reasons, "samples": len(inside)}


def physical_gpu(local_rank: int) -> str:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


# ------------------------------------------------------------------ reference CPU workers


def _ref_worker(rows, setup_q, go, result_q, steps):
    """One host process running MiniXLA's execute() on `rows` of the 8192^3 workload."""
    sys.path.insert(0, str(ROOT))
    from minixla_b200 import datagen
    from oracle.bindings import REF_LIB, RefGraph, fused_oracle

    kind = "reference" if REF_LIB.exists() else "port"
    B = datagen.uniform((NDIM, NDIM), 1)
    A = datagen.uniform((len(rows), NDIM), 0, row_offset=rows[0])
    Cm = datagen.normal((len(rows), NDIM), 2, row_offset=rows[0])
    if kind == "reference":
        rg = RefGraph()
        L = rg.lib
        root = rg.optimize(L.g_relu(L.g_add(L.g_matmul(rg.input(A), rg.input(B)), rg.input(Cm))))
        del B

        def run():
            node = root.contents
            if node.owns_output and node.output:
                L.free_tensor(node.output)     # drop the memoized result (bench.c:230-231)
            node.output = None
            node.owns_output = 0
            if not L.execute(root):
                raise RuntimeError("execute() failed")
    else:
        def run():
            fused_oracle(A, B, [("add", Cm), ("relu",)], threads=1)
    setup_q.put(kind)
    for _ in range(steps):
        go.wait()
        t0 = time.perf_counter()
        run()
        result_q.put(time.perf_counter() - t0)


def run_reference_steps(total_steps: int, rows_per_worker: int, workers: int):
    """Runs `total_steps` synchronized steps over `workers` processes; returns
    (per-step wall seconds, rows per step, kind)."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    go = ctx.Barrier(workers + 1)
    setup_q, result_q = ctx.Queue(), ctx.Queue()
    procs = []
    for w in range(workers):
        r0 = w * (ROWS_PER_GPU // workers)
        rows = list(range(r0, r0 + rows_per_worker))
        p = ctx.Process(target=_ref_worker, args=(rows, setup_q, go, result_q, total_steps), daemon=True)
        p.start()
        procs.append(p)
    kinds = {setup_q.get(timeout=600) for _ in range(workers)}
    walls = []
    for _ in range(total_steps):
        t0 = time.perf_counter()
        go.wait()
        for _ in range(workers):
            result_q.get(timeout=3600)
        walls.append(time.perf_counter() - t0)
    for p in procs:
        p.join(timeout=60)
    return walls, rows_per_worker * workers, ("reference" if kinds == {"reference"} else "port")


def host_workers() -> int:
    return max(1, min(os.cpu_count() or 1, 16))


def cpu_baseline(rows_target: int = 16):
    workers = host_workers()
    rpw = max(1, round(rows_target / workers))
    walls, rows, kind = run_reference_steps(2, rpw, workers)
    wall = walls[-1]
    tflops = 2.0 * rows * NDIM * NDIM / wall / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": workers, "kind": kind,
            "sample": f"{rows} output rows of relu(A.B+C) at K=N=8192 ({rpw} per process, {workers} processes "
                      f"in parallel) through MiniXLA's execute(); second of two timed passes; "
                      f"{wall:.2f} s wall"}


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    workers = host_workers()
    walls, rows, kind = run_reference_steps(args.warmup + args.steps, 1, workers)
    timed = walls[args.warmup:]
    total = sum(timed)
    value = 2.0 * rows * len(timed) * NDIM * NDIM / total / 1e12
    line = {
        "metric": "fused relu(A.B+C) TFLOP/s (fp32 in/out)", "impl": "reference", "value": value,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "devices": "host CPU cores only (the reference's execute())",
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / len(timed), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded splitmix64: A,B ~ U[-1,1], C ~ N(0,1))",
        "config": {"workload": "relu(A.B+C) 8192x8192x8192 per shard, row sample per step",
                   "rows_per_step": rows, "N": NDIM, "K": NDIM, "parallelism": f"{workers} host processes",
                   "note": "host CPU cores only: the reference's execute() has no GPU or multi-GPU path, so this "
                           "value is the same at every N"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": workers, "kind": kind,
                         "sample": f"{rows} output rows per step ({workers} processes x 1 row) through "
                                   "MiniXLA's execute()"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ our arm


def measured_hbm_gbs():
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(f.read_text())["hbm_gbs"])
        return v, f"measured copy {v:.1f} GB/s (MEASURED_PEAKS.json)"
    except Exception:
        return 6650.0, "fallback copy 6650 GB/s"


def measured_tf32_peak(sustained: bool = False):
    """TF32 dense peak: the measured bf16 GEMM rate of this pool halved (TF32
    tensor-core math runs at half the bf16 rate on B200) -- the burst figure,
    or the seconds-long power-capped one with sustained=True."""
    f = ROOT / "MEASURED_PEAKS.json"
    key, label = ("bf16_tflops_sustained", "sustained") if sustained else ("bf16_tflops", "burst")
    try:
        bf16 = float(json.loads(f.read_text())[key])
        return bf16 / 2.0, f"measured bf16 {label} {bf16:.1f} TFLOP/s / 2 (MEASURED_PEAKS.json)"
    except Exception:
        v = 1400.0 if sustained else 1590.0
        return v / 2.0, f"fallback bf16 {label} {v:.0f} TFLOP/s / 2"


SPEC_TF32_TFLOPS = 1125.0  # B200 nominal dense TF32 (half the 2.25 PFLOP/s dense bf16 figure)


def time_allgather(out_d, world, m_total, stream, warmup, steps, max_over_ranks):
    """NCCL all-gather of every rank's [M, N] output rows into [m_total, N] on
    the bench stream: mean CUDA-event time per gather, max over ranks.  Every
    rank runs the same number of gathers."""
    import torch
    import torch.distributed as dist

    M, N = out_d.shape
    full = torch.empty((m_total, N), device=out_d.device, dtype=out_d.dtype)
    equal = M * world == m_total
    with torch.cuda.stream(stream):
        if equal:
            def gather():
                dist.all_gather_into_tensor(full, out_d)
        else:
            sizes = [torch.zeros(1, device=out_d.device, dtype=torch.int64) for _ in range(world)]
            dist.all_gather(sizes, torch.tensor([M], device=out_d.device, dtype=torch.int64))
            parts = list(torch.split(full, [int(s.item()) for s in sizes]))

            def gather():
                dist.all_gather([p for p in parts], out_d)
        for _ in range(max(1, warmup)):
            gather()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            gather()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    total_bytes = 4.0 * m_total * N
    recv = total_bytes - 4.0 * M * N
    return {"ms_per_step": ms, "bytes_gathered": int(total_bytes), "bytes_received_per_gpu": int(recv),
            "algbw_GBs": total_bytes / (ms * 1e-3) / 1e9,
            "busbw_GBs": total_bytes * (world - 1) / world / (ms * 1e-3) / 1e9,
            "collective": "torch.distributed all_gather_into_tensor (NCCL)", "in_value": False}, full


def time_fused_allgather(lib, ctx, local_rank, A_d, B_d, steps_arr, r0, M, N, K, m_total, prec, stream, warmup,
                         steps, max_over_ranks, ref_full):
    """The fused form of the same gather: each step is one
    mxb_fused_gemm_allgather (the kernel writes this rank's rows into every
    rank's full buffer over NVLink) plus the one-element all-reduce a reader
    needs before it reads peer rows.  Mean CUDA-event time per step, max over
    ranks; the full buffer is compared bit for bit with the NCCL gather of
    the separately computed rows."""
    import torch
    import torch.distributed as dist

    from minixla_b200 import lib as mlib
    from minixla_b200.peer_gather import GatherBuffers

    gb = GatherBuffers(lib, local_rank, m_total, N)
    try:
        def step():
            rc = gb.gemm(ctx, A_d.data_ptr(), K, B_d.data_ptr(), N, r0, M, N, K, steps_arr, 2, prec,
                         stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"mxb_fused_gemm_allgather failed: {mlib.last_error()}")
            gb.barrier(stream)

        for _ in range(max(1, warmup)):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        pushes0 = lib.mxb_gather_push_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        in_kernel = max_over_ranks(0.0 if lib.mxb_gather_push_count() - pushes0 == steps else 1.0) == 0.0
        exact = max_over_ranks(0.0 if torch.equal(gb.tensor(), ref_full) else 1.0) == 0.0
    finally:
        gb.close()
    world = dist.get_world_size()
    return {"ms_per_step": ms, "rows_written_by_kernel": in_kernel, "bit_equal_to_nccl_gather": exact,
            "peer_GBs_per_direction": 4.0 * M * N * (world - 1) / (ms * 1e-3) / 1e9,
            "form": "mxb_fused_gemm_allgather: epilogue stores to CUDA-IPC peer buffers over NVLink, "
                    "+ one-element NCCL all-reduce per step"}


def traffic_from_profile(precision: str, m: int):
    f = ROOT / "profiles" / f"fused_gemm_{precision}_{ROWS_PER_GPU}.json"
    try:
        d = json.loads(f.read_text())
        return float(d["dram_bytes_per_launch"]) * m / float(d["rows"])
    except Exception:
        return None


def check_rows(M: int, r0: int, n_random: int = 48, seed: int = 0):
    """Rows of a shard [r0, r0 + M) to check against the oracle: the shard's
    edges, the CTA-pair tile edges (every 256 rows of the job, and the first
    ones inside the shard), and random rows."""
    import numpy as np

    rows = {0, 1, M // 2, M - 2, M - 1, 127, 128, 255, 256, 257}
    first = (r0 + 255) // 256 * 256
    for g in range(first, r0 + M, 256 * max(1, M // (256 * 8))):
        rows.update({g - r0 - 1, g - r0})
    rng = np.random.default_rng(seed + r0)
    rows.update(rng.integers(0, M, n_random).tolist())
    return sorted(r for r in rows if 0 <= r < M)


def time_steps(launch, stream, warmup: int, steps: int) -> float:
    """Mean CUDA-event time of `steps` back-to-back launches on `stream`, after `warmup`."""
    import torch

    for _ in range(warmup):
        launch()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def strong_leg(args, lib, ctx, dev, stream, rank, local_rank, world, prec, B_h, B_d, max_over_ranks, barrier, tol):
    """The fixed 32768 x 8192 x 8192 relu(A.B + C) job split by rows over the
    N GPUs: kernel-only time (max over ranks), the same with the row
    all-gather -- fused into the epilogue (mxb_fused_gemm_allgather) and as an
    NCCL all-gather after the kernel -- and the 1-GPU time of the whole job
    (rank 0 alone, the others waiting), from which speed-up and efficiency
    follow.  Every rank checks >= 64 rows of its shard against the oracle."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from minixla_b200 import datagen
    from minixla_b200 import lib as mlib
    from oracle.bindings import fused_oracle

    N = K = NDIM
    m_total = STRONG_M
    r0, r1, _ = shard_rows(world, rank, "strong")
    M = r1 - r0
    flops_job = 2.0 * m_total * N * K

    def steps_for(C_dev):
        st = (mlib.EpStepDev * 2)()
        st[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, C_dev.data_ptr(), N, 0.0, 0)
        st[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
        return st

    def gemm_launcher(A_dev, C_dev, out_dev, rows):
        st = steps_for(C_dev)

        def launch():
            rc = lib.mxb_fused_gemm(ctx, A_dev.data_ptr(), K, B_d.data_ptr(), N, out_dev.data_ptr(), N, rows, N, K,
                                    st, 2, prec, stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"mxb_fused_gemm failed: {mlib.last_error()}")
        return launch, st

    # The whole job on one GPU (rank 0; at N = 1 this is the shard itself).
    one_gpu_ms = None
    if world > 1:
        if rank == 0:
            A_f = torch.from_numpy(datagen.uniform((m_total, K), 0)).to(dev)
            C_f = torch.from_numpy(datagen.normal((m_total, N), 2)).to(dev)
            O_f = torch.empty((m_total, N), device=dev)
            launch_f, _ = gemm_launcher(A_f, C_f, O_f, m_total)
            one_gpu_ms = time_steps(launch_f, stream, max(3, args.warmup), args.steps)
            del A_f, C_f, O_f
            torch.cuda.empty_cache()
        barrier()
        t = torch.tensor([one_gpu_ms or 0.0], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        one_gpu_ms = float(t.item())

    A_h = datagen.uniform((M, K), 0, row_offset=r0)
    C_h = datagen.normal((M, N), 2, row_offset=r0)
    A_s, C_s = torch.from_numpy(A_h).to(dev), torch.from_numpy(C_h).to(dev)
    out_s = torch.empty((M, N), device=dev)
    launch_s, st_s = gemm_launcher(A_s, C_s, out_s, M)
    barrier()
    shard_ms = max_over_ranks(time_steps(launch_s, stream, max(3, args.warmup), args.steps))
    if world == 1:
        one_gpu_ms = shard_ms

    rows = check_rows(M, r0)
    want = fused_oracle(A_h, B_h, [("add", C_h), ("relu",)], rows=rows)
    got = out_s[rows].cpu().numpy()
    rel = max_over_ranks(float(np.linalg.norm(got - want) / np.linalg.norm(want)))
    if not rel <= tol:
        raise RuntimeError(f"strong-scaling result check failed: relative error {rel:.3g} > {tol}")
    n_rows = int(max_over_ranks(-len(rows)) * -1)  # fewest rows checked on any rank

    def entry(ms):
        return {"ms_per_step": ms, "tflops": flops_job / (ms * 1e-3) / 1e12,
                "speedup_vs_1gpu": one_gpu_ms / ms, "efficiency": one_gpu_ms / ms / world}

    out = {
        "workload": "relu(A.B+C) 32768x8192x8192 split by rows over N GPUs (mxb_shard_rows)",
        "rows_per_gpu": M, "one_gpu_ms": one_gpu_ms,
        "one_gpu_tflops": flops_job / (one_gpu_ms * 1e-3) / 1e12,
        "kernel": entry(shard_ms),
        "kernel_efficiency": one_gpu_ms / shard_ms / world,
        "speedup_vs_1gpu": one_gpu_ms / shard_ms,
        "streamk_tiles_per_gpu": mlib.gemm_plan(M, N, K, prec, torch.cuda.get_device_properties(dev)
                                                .multi_processor_count).streamk_tiles,
        "check": {"rows_per_rank": n_rows, "rel_err_max_over_ranks": rel, "tol": tol,
                  "rows": "shard edges, 256-row tile edges, 48 random rows per rank; oracle (eval_fused restated)"},
        "gather_nccl": None, "gather_fused": None,
    }
    if world > 1:
        ag, gathered = time_allgather(out_s, world, m_total, stream, args.warmup, args.steps, max_over_ranks)
        out["gather_nccl"] = entry(shard_ms + ag["ms_per_step"])
        out["gather_nccl"].update({"allgather_ms": ag["ms_per_step"], "busbw_GBs": ag["busbw_GBs"],
                                   "form": "kernel, then torch.distributed all_gather (NCCL)"})
        fused = time_fused_allgather(lib, ctx, local_rank, A_s, B_d, st_s, r0, M, N, K, m_total, prec, stream,
                                     args.warmup, args.steps, max_over_ranks, gathered)
        out["gather_fused"] = entry(fused["ms_per_step"])
        out["gather_fused"].update({k: fused[k] for k in ("rows_written_by_kernel", "bit_equal_to_nccl_gather",
                                                          "form", "peer_GBs_per_direction")})
        del gathered
    del A_s, C_s, out_s
    torch.cuda.empty_cache()
    return out


def sharded_executor_leg(lib, world, prec, tol, reps: int = 2):
    """One process driving all N GPUs through the product's own multi-GPU
    executor (gpu_ctx_create_multi + gpu_execute): the 32768 x 8192 x 8192
    relu(A.B + C) node on pageable host buffers, rows split over the GPUs,
    B replicated by peer copies; host-clock time per call (inputs up, result
    down, as a MiniXLA caller sees it) and sampled rows against the oracle."""
    import numpy as np

    from minixla_b200 import datagen
    from minixla_b200 import lib as mlib
    from minixla_b200.abi import OP_ADD, OP_RELU, HostGraph, free_host_tensor
    from oracle.bindings import fused_oracle

    N = K = NDIM
    M = STRONG_M
    A = datagen.uniform((M, K), 0)
    B = datagen.uniform((K, N), 1)
    Cm = datagen.normal((M, N), 2)
    ctx = lib.gpu_ctx_create_multi(world)
    if not ctx:
        raise RuntimeError(f"gpu_ctx_create_multi({world}) failed: {mlib.last_error()}")
    try:
        lib.gpu_ctx_set_precision(ctx, prec)
        hg = HostGraph()
        root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(Cm)), (OP_RELU, None)])
        rows = sorted(set(check_rows(M, 0, 40)) | {g * (M // world) + d for g in range(1, world) for d in (-1, 0)})
        ts = []
        got = None
        for i in range(reps + 1):
            t0 = time.perf_counter()
            t = lib.gpu_execute(root, ctx)
            if not t:
                raise RuntimeError(f"sharded gpu_execute failed: {mlib.last_error()}")
            if i == reps:
                # only the checked rows: a copy of the whole 1 GiB result would land in the timing
                got = np.ctypeslib.as_array(t.contents.data, shape=(M * N,)).reshape(M, N)[rows].copy()
            free_host_tensor(t)
            if i > 0:
                ts.append(time.perf_counter() - t0)
        ngpu = lib.gpu_ctx_ngpu(ctx)
    finally:
        lib.gpu_ctx_destroy(ctx)
    want = fused_oracle(A, B, [("add", Cm), ("relu",)], rows=rows)
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    if not rel <= tol:
        raise RuntimeError(f"sharded executor check failed: relative error {rel:.3g} > {tol}")
    ms = 1e3 * min(ts)
    return {"entry_point": "gpu_ctx_create_multi + gpu_execute (pageable host buffers)", "gpus": ngpu,
            "workload": "relu(A.B+C) 32768x8192x8192", "ms": ms, "ms_all": [1e3 * x for x in ts],
            "tflops_end_to_end": 2.0 * M * N * K / (ms * 1e-3) / 1e12, "rel_err": rel, "tol": tol,
            "rows_checked": len(rows), "h2d_bytes": 4 * (M * K + K * N + M * N), "d2h_bytes": 4 * M * N}


def ours_arm(args, rank, local_rank, world):
    import numpy as np
    import torch
    import torch.distributed as dist

    from minixla_b200 import datagen
    from minixla_b200 import lib as mlib
    from minixla_b200.abi import OP_ADD, OP_RELU, HostGraph, free_host_tensor

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=dt.timedelta(seconds=300), device_id=dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # CPU baseline first, before this process touches its GPU (rank 0, one GPU).
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline()

    lib = mlib.load()
    prec = mlib.GPU_PRECISION_TF32 if args.precision == "tf32" else mlib.GPU_PRECISION_3XTF32
    r0, r1, m_total = shard_rows(world, rank, args.workload, args.shape)
    M = r1 - r0
    N = K = args.shape or NDIM
    A = datagen.uniform((M, K), 0, row_offset=r0)
    B = datagen.uniform((K, N), 1)
    Cm = datagen.normal((M, N), 2, row_offset=r0)
    tol = 2e-3 if prec == mlib.GPU_PRECISION_TF32 else 1e-5

    ctx = lib.gpu_ctx_create_on(local_rank)
    if not ctx:
        raise RuntimeError(f"gpu_ctx_create_on({local_rank}) failed: {mlib.last_error()}")
    lib.gpu_ctx_set_precision(ctx, prec)

    # ---- device-resident timing (value)
    A_d, B_d, C_d = (torch.from_numpy(x).to(dev) for x in (A, B, Cm))
    out_d = torch.empty((M, N), device=dev, dtype=torch.float32)
    steps = (mlib.EpStepDev * 2)()
    steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, C_d.data_ptr(), N, 0.0, 0)
    steps[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
    # A dedicated stream: torch's default stream has handle 0, which the C ABI
    # reads as "the context's own stream", and the events must sit on the
    # stream the kernels run on.
    stream = torch.cuda.Stream(dev)

    def launch(p=prec):
        rc = lib.mxb_fused_gemm(ctx, A_d.data_ptr(), K, B_d.data_ptr(), N, out_d.data_ptr(), N, M, N, K, steps, 2,
                                p, stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(f"mxb_fused_gemm failed: {mlib.last_error()}")

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    if lib.mxb_check_device_error(ctx) != 0:
        raise RuntimeError(mlib.last_error())

    sampler = ClockSampler(physical_gpu(local_rank))
    sampler.start()
    ev_s = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev_e = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    launches0 = lib.mxb_launch_count()
    h0 = time.time()
    t_start.record(stream)
    for i in range(args.steps):
        ev_s[i].record(stream)
        launch()
        ev_e[i].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    h1 = time.time()
    launches = lib.mxb_launch_count() - launches0
    barrier()
    clocks = sampler.stop(h0, h1)
    if lib.mxb_check_device_error(ctx) != 0:
        raise RuntimeError(mlib.last_error())
    total_ms = max_over_ranks(t_start.elapsed_time(t_end))
    per_launch_ms = statistics.mean(ev_s[i].elapsed_time(ev_e[i]) for i in range(args.steps))
    per_launch_ms = max_over_ranks(per_launch_ms)

    flops_rank = 2.0 * M * N * K
    flops_job = 2.0 * m_total * N * K
    value = flops_job * args.steps / (total_ms * 1e-3) / 1e12

    # spot check of this rank's result against the oracle on a few rows
    from oracle.bindings import fused_oracle

    rows = [0, M // 2, M - 1]
    want = fused_oracle(A, B, [("add", Cm), ("relu",)], rows=rows)
    got = out_d[rows].cpu().numpy()
    rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    if not rel <= tol:
        raise RuntimeError(f"bench result check failed: relative error {rel:.3g} > {tol}")

    # All-gather of the output rows over NVLink (N > 1): timed separately, as
    # the row-sharded job only needs it when a consumer wants the full tensor.
    allgather = None
    if world > 1:
        allgather, gathered = time_allgather(out_d, world, m_total, stream, args.warmup, args.steps, max_over_ranks)
        allgather["kernel_plus_allgather_tflops"] = flops_job / (
            (total_ms / args.steps + allgather["ms_per_step"]) * 1e-3) / 1e12
        fused = time_fused_allgather(lib, ctx, local_rank, A_d, B_d, steps, r0, M, N, K, m_total, prec, stream,
                                     args.warmup, args.steps, max_over_ranks, gathered)
        fused["kernel_plus_allgather_tflops"] = flops_job / (fused["ms_per_step"] * 1e-3) / 1e12
        allgather["fused"] = fused
        del gathered

    # ---- the default precision (3xTF32, fp32-faithful) through the same timed loop
    x3 = None
    if prec == mlib.GPU_PRECISION_TF32 and not args.shape:
        sampler3 = ClockSampler(physical_gpu(local_rank))
        sampler3.start()
        h3 = time.time()
        ms3 = max_over_ranks(time_steps(lambda: launch(mlib.GPU_PRECISION_3XTF32), stream, max(3, args.warmup),
                                        args.steps))
        clocks3 = sampler3.stop(h3, time.time())
        rows3 = check_rows(M, r0, 13)
        want3 = fused_oracle(A, B, [("add", Cm), ("relu",)], rows=rows3)
        rel3 = max_over_ranks(float(np.linalg.norm(out_d[rows3].cpu().numpy() - want3) / np.linalg.norm(want3)))
        if not rel3 <= 1e-5:
            raise RuntimeError(f"3xTF32 result check failed: relative error {rel3:.3g} > 1e-5")
        pk3, pk3_src = measured_tf32_peak()
        pk3s, pk3s_src = measured_tf32_peak(sustained=True)
        ach3 = flops_rank / (ms3 * 1e-3) / 1e12
        x3 = {"value": flops_job / (ms3 * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms3,
              "steps": args.steps, "rel_err_rows": rel3, "rows_checked": len(rows3), "tol": 1e-5,
              "roofline": {"bound": "tensor", "achieved": ach3, "peak": pk3 / 3.0, "unit": "TFLOP/s",
                           "frac": ach3 / (pk3 / 3.0),
                           "peak_source": pk3_src + " / 3 (three TF32 products per multiply-add)",
                           "peak_sustained": pk3s / 3.0, "frac_of_sustained": ach3 / (pk3s / 3.0),
                           "peak_sustained_source": pk3s_src + " / 3"},
              "clocks": clocks3,
              "note": "gpu_execute's default mode: x = big + small, three TF32 products, segment sums in fp32; "
                      "the timed call includes the pre-pass that writes the low parts of A and B"}

    # cuBLAS TF32 on the same shape, for context only (not on the product path):
    # the same number of back-to-back steps, so both run under the same power
    # cap, and the best of 10 single launches as the measured TF32 peak.
    cublas = cublas_best = None
    if rank == 0:
        torch.backends.cuda.matmul.allow_tf32 = True
        with torch.cuda.stream(stream):
            ref_out = torch.empty_like(out_d)
            for _ in range(args.warmup):
                torch.matmul(A_d, B_d, out=ref_out)
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            for _ in range(args.steps):
                torch.matmul(A_d, B_d, out=ref_out)
            c1.record(stream)
            torch.cuda.synchronize()
            cublas = flops_rank * args.steps / (c0.elapsed_time(c1) * 1e-3) / 1e12
            singles = []
            for _ in range(10):
                c0.record(stream)
                torch.matmul(A_d, B_d, out=ref_out)
                c1.record(stream)
                torch.cuda.synchronize()
                singles.append(c0.elapsed_time(c1))
            cublas_best = flops_rank / (min(singles) * 1e-3) / 1e12
        torch.backends.cuda.matmul.allow_tf32 = False
        del ref_out

    # ---- the fixed 32768 x 8192 x 8192 job split over the N GPUs (strong scaling)
    strong = None
    if not args.shape and not args.no_strong:
        strong = strong_leg(args, lib, ctx, dev, stream, rank, local_rank, world, prec, B, B_d, max_over_ranks,
                            barrier, tol)
    del out_d
    torch.cuda.empty_cache()

    # ---- end to end through the reference-facing C ABI
    e2e = None
    if not args.no_e2e:
        h2d = 4 * (M * K + K * N + M * N)
        d2h = 4 * M * N
        # Headline: gpu_execute, exactly as a MiniXLA program calls it -- the
        # inputs in pageable (malloc'd) host memory as create_tensor leaves
        # them, a fresh result tensor returned and released with free_tensor's
        # frees, every step.
        hp = HostGraph()
        root_p = hp.fused_node(hp.input_node(A), hp.input_node(B), [(OP_ADD, hp.input_node(Cm)), (OP_RELU, None)])

        def execute_once():
            t = lib.gpu_execute(root_p, ctx)
            if not t:
                raise RuntimeError(f"gpu_execute failed: {mlib.last_error()}")
            return t

        for _ in range(2):
            free_host_tensor(execute_once())
        barrier()
        ts = []
        last = None
        for i in range(args.e2e_steps):
            t0 = time.perf_counter()
            t = execute_once()
            if i == args.e2e_steps - 1:
                last = np.ctypeslib.as_array(t.contents.data, shape=(M * N,)).reshape(M, N)[rows].copy()
            free_host_tensor(t)
            ts.append(time.perf_counter() - t0)
        g_ms = max_over_ranks(1e3 * statistics.mean(ts))
        rel_e2e = float(np.linalg.norm(last - want) / np.linalg.norm(want))
        if not rel_e2e <= tol:
            raise RuntimeError(f"e2e result check failed: relative error {rel_e2e:.3g} > {tol}")
        e2e = {"value": flops_job / (g_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": g_ms,
               "steps": args.e2e_steps, "entry_point": "gpu_execute (pageable malloc'd host buffers; the returned "
                                                       "tensor freed inside the step)",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

        # The additive gpu_execute_into with pinned host buffers (the copies at
        # full link speed).
        A_h = torch.from_numpy(A).pin_memory()
        B_h = torch.from_numpy(B).pin_memory()
        C_h = torch.from_numpy(Cm).pin_memory()
        O_h = torch.empty((M, N), dtype=torch.float32).pin_memory()
        hg = HostGraph()
        root = hg.fused_node(hg.input_node(A_h), hg.input_node(B_h),
                             [(OP_ADD, hg.input_node(C_h)), (OP_RELU, None)])
        out_t = hg.tensor(O_h)

        def timed_into(r, o):
            for _ in range(2):
                if lib.gpu_execute_into(r, ctx, o) != 0:
                    raise RuntimeError(mlib.last_error())
            barrier()
            e0 = time.perf_counter()
            for _ in range(args.e2e_steps):
                if lib.gpu_execute_into(r, ctx, o) != 0:
                    raise RuntimeError(mlib.last_error())
            return max_over_ranks((time.perf_counter() - e0) * 1e3 / args.e2e_steps)

        e_ms = timed_into(root, out_t)
        rel_into = float(np.linalg.norm(O_h[rows].numpy() - want) / np.linalg.norm(want))
        if not rel_into <= tol:
            raise RuntimeError(f"e2e (pinned) result check failed: relative error {rel_into:.3g} > {tol}")
        e2e["pinned_into"] = {"value": flops_job / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e_ms,
                              "entry_point": "gpu_execute_into (pinned host buffers)",
                              "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        # Same, with B kept resident on the GPU (weights that stay between calls):
        # A and C still go up and the result comes down every step.
        b_tensor = root.contents.inputs[1].contents.output
        if lib.gpu_ctx_keep_resident(ctx, b_tensor) != 0:
            raise RuntimeError(mlib.last_error())
        r_ms = timed_into(root, out_t)
        lib.gpu_ctx_release_resident(ctx, None)
        e2e["b_resident"] = {"value": flops_job / (r_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": r_ms,
                             "h2d_bytes_per_step": 4 * (M * K + M * N), "d2h_bytes_per_step": d2h,
                             "note": "gpu_execute_into, pinned, B kept resident with gpu_ctx_keep_resident"}

        # gpu_execute_into with pageable buffers: through the context's pinned
        # staging slots, and with staging off (the driver's own pageable path).
        out_p = np.empty((M, N), dtype=np.float32)
        out_pt = hp.tensor(out_p)
        pageable = {}
        # The driver's own pageable path is slow (~90 ms a step on one GPU):
        # measured on one GPU only.
        for label, staged in (("staged", "1"), ("driver_copy", "0"))[: 2 if world == 1 else 1]:
            os.environ["MINIXLA_STAGED_COPY"] = staged
            p_ms = timed_into(root_p, out_pt)
            pageable[label] = {"value": flops_job / (p_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": p_ms}
        os.environ.pop("MINIXLA_STAGED_COPY", None)
        if not np.array_equal(out_p, O_h.numpy()):
            raise RuntimeError("pageable e2e result differs from the pinned one")
        pageable["note"] = ("gpu_execute_into on pageable host buffers: 'staged' copies through the context's "
                            "pinned slots filled by several host threads; 'driver_copy' is the CUDA driver's own "
                            "pageable path (MINIXLA_STAGED_COPY=0)")
        e2e["pageable_into"] = pageable
        e2e["vs_pinned_into"] = g_ms / e_ms

    peak, peak_src = measured_tf32_peak()
    if prec == mlib.GPU_PRECISION_3XTF32:
        peak, peak_src = peak / 3.0, peak_src + " / 3 (three TF32 products per multiply-add)"
    achieved = flops_rank / (per_launch_ms * 1e-3) / 1e12
    lib.gpu_ctx_destroy(ctx)

    # Ranks meet once more, then leave; rank 0 alone drives all N GPUs
    # through the product's multi-GPU executor.
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    sharded = None
    if world > 1 and not args.shape and not args.no_strong:
        torch.cuda.synchronize()
        sharded = sharded_executor_leg(lib, world, prec, tol)

    spec = SPEC_TF32_TFLOPS / (3.0 if prec == mlib.GPU_PRECISION_3XTF32 else 1.0)
    line = {
        "metric": "fused relu(A.B+C) TFLOP/s (fp32 in/out)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.workload in ("strong", "config5") else "weak",
        "vs_baseline": None, "dtype": args.precision,
        "data": "synthetic (seeded splitmix64: A,B ~ U[-1,1], C ~ N(0,1))",
        "config": {
            "workload": ("relu(A.B+C) 32768x8192x8192 split over N GPUs" if args.workload in ("strong", "config5")
                         else "relu(A.B+C) 8192x8192x8192 per GPU (8192-row shard each)"),
            "M_total": m_total, "N": N, "K": K, "rows_per_gpu": M, "precision": args.precision,
            "parallelism": f"row-shard x{world}",
            "l2": "inputs larger than L2 (A+B+C = 768 MiB per GPU step), no flush",
        },
        "gpu_launches": int(launches),
        "e2e": e2e,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic_from_profile(args.precision, M),
                     "peak_source": peak_src, "kernel_ms": per_launch_ms,
                     "frac_of_spec": achieved / spec, "spec_peak": "1125 TFLOP/s dense TF32 (B200 nominal)",
                     "peak_cublas_tf32_best_of_10": cublas_best if prec == mlib.GPU_PRECISION_TF32 else None,
                     "frac_of_cublas_tf32_best_of_10": (achieved / cublas_best)
                     if cublas_best and prec == mlib.GPU_PRECISION_TF32 else None,
                     "frac_of_cublas_tf32": (achieved / cublas) if cublas and prec == mlib.GPU_PRECISION_TF32
                     else None},
        "precision_3xtf32": x3,
        "strong": strong,
        "sharded_executor": sharded,
        "allgather": allgather,
        "cpu_baseline": cpu,
        "clocks": clocks,
        "cublas_tf32_matmul_tflops_same_shape_same_steps": cublas,
        "result_check_rel_err": rel,
    }
    print(json.dumps(line), flush=True)
    return 0


SWEEP_SHAPES = [  # (M, N, K, C distribution) -- the benchmark workloads: 128^3, the square sweep, the ragged shapes, 32768 x 8192 x 8192 on one GPU
    (128, 128, 128, "uniform"),
    (512, 512, 512, "normal"), (1024, 1024, 1024, "normal"), (2048, 2048, 2048, "normal"),
    (4096, 4096, 4096, "normal"), (8192, 8192, 8192, "normal"),
    (1000, 1000, 1000, "uniform"), (257, 4097, 129, "uniform"), (8191, 127, 3000, "uniform"),
    (1, 4096, 4096, "uniform"), (32768, 8192, 8192, "normal"),
]


CPU_SLICE_FLOPS = 0.3e9  # per reference timing: about 0.3 s of single-threaded execute()


def cpu_reference_ms(build, rows_total: int, flops_per_row: float):
    """Single-threaded wall time of MiniXLA's own execute() (oracle/_ref) for
    a graph over `rows_total` output rows, from a timed row slice: rows are
    independent through eval_fused, so the time scales linearly in M.
    `build(rg, r)` builds the graph of the first r rows with RefGraph and
    returns its root.  Falls back to the C restatement when the reference
    library is absent (kind "port")."""
    from oracle.bindings import RefGraph, ref_available

    r = int(max(1, min(rows_total, CPU_SLICE_FLOPS // max(1.0, flops_per_row))))
    if not ref_available():
        return {"cpu_reference_ms": None, "cpu_kind": "unavailable"}
    rg = RefGraph()
    try:
        root = rg.own(rg.optimize(build(rg, r)))
        t0 = time.perf_counter()
        rg.execute(root)
        dt = time.perf_counter() - t0
    finally:
        rg.close()
    return {"cpu_reference_ms": dt * 1e3 * rows_total / r, "cpu_rows_timed": r,
            "cpu_extrapolated": r < rows_total, "cpu_kind": "reference execute(), 1 thread"}


def run_sweep(args):
    """Kernel-only time of relu(A.B + C) for every benchmark shape, both
    precision modes, operands resident (min and median of CUDA-event-timed
    launches after warm-up; each behind a ~50 us spin on the stream so the
    host's launch preparation stays outside the events), plus the 3-layer
    3-layer MLP DAG (X 4096 x 1024, hidden 4096) through the device API (one
    launch per fused node)."""
    import numpy as np
    import torch

    from minixla_b200 import datagen
    from minixla_b200 import lib as mlib

    lib = mlib.load()
    ctx = lib.gpu_ctx_create_on(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    peak, _ = measured_tf32_peak()

    def pad4(x):
        # TMA needs 16-byte row pitches: pad the columns as gpu_execute does.
        cols = x.shape[1]
        if cols % 4 == 0:
            return x, cols
        p = torch.zeros((x.shape[0], (cols + 3) // 4 * 4), device=dev)
        p[:, :cols] = x
        return p, p.shape[1]

    def time_launches(fn, reps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # Keep the stream busy (~50 us) while the call is prepared, so the
            # events bracket the kernels rather than the host's launch work.
            with torch.cuda.stream(stream):
                torch.cuda._sleep(100_000)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return min(ts), statistics.median(ts)

    shapes = SWEEP_SHAPES
    if args.mnk:
        m, n, k = (int(v) for v in args.mnk.split(","))
        shapes = [(m, n, k, "uniform")]
    for M, N, K, cdist in shapes:
        A = torch.from_numpy(datagen.uniform((M, K), 0)).to(dev)
        B = torch.from_numpy(datagen.uniform((K, N), 1)).to(dev)
        Cm = torch.from_numpy(datagen.normal((M, N), 2) if cdist == "normal" else datagen.uniform((M, N), 2)).to(dev)
        out = torch.empty((M, N), device=dev)
        Ap, lda = pad4(A)
        Bp, ldb = pad4(B)
        steps = (mlib.EpStepDev * 2)()
        steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, Cm.data_ptr(), N, 0.0, 0)
        steps[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)
        flops = 2.0 * M * N * K
        algo_bytes = 4.0 * (M * K + K * N + 2 * M * N)
        A_h, B_h, C_h = A.cpu().numpy(), B.cpu().numpy(), Cm.cpu().numpy()

        def build_rows(rg, r, A_h=A_h, B_h=B_h, C_h=C_h):
            L = rg.lib
            return L.g_relu(L.g_add(L.g_matmul(rg.input(A_h[:r]), rg.input(B_h)), rg.input(C_h[:r])))

        cpu = None if args.no_cpu_baseline else cpu_reference_ms(build_rows, M, 2.0 * N * K)
        del A_h, B_h, C_h
        for prec_name, prec in (("tf32", mlib.GPU_PRECISION_TF32), ("3xtf32", mlib.GPU_PRECISION_3XTF32)):
            def fn():
                rc = lib.mxb_fused_gemm(ctx, Ap.data_ptr(), lda, Bp.data_ptr(), ldb, out.data_ptr(), N, M, N, K,
                                        steps, 2, prec, stream.cuda_stream)
                assert rc == 0, mlib.last_error()
            reps = 20 if flops < 1e12 else 5
            tmin, tmed = time_launches(fn, reps)
            pk = peak if prec == mlib.GPU_PRECISION_TF32 else peak / 3
            line = {"sweep": "fused relu(A.B+C)", "M": M, "N": N, "K": K, "precision": prec_name,
                    "ms_min": tmin, "ms_median": tmed, "tflops": flops / (tmin * 1e-3) / 1e12,
                    "frac_tensor_peak": flops / (tmin * 1e-3) / 1e12 / pk,
                    "gbs": algo_bytes / (tmin * 1e-3) / 1e9}
            if cpu:
                line.update(cpu)
                if cpu.get("cpu_reference_ms"):
                    line["speedup_vs_cpu_reference"] = cpu["cpu_reference_ms"] / tmin
            print(json.dumps(line), flush=True)
        del A, B, Cm, out, Ap, Bp
        torch.cuda.empty_cache()

    if args.mnk:
        lib.gpu_ctx_destroy(ctx)
        return 0
    # the 3-layer MLP, one launch per fused node (+ the bare matmul)
    Mx, D, H = 4096, 1024, 4096
    X = torch.from_numpy(datagen.uniform((Mx, D), 70)).to(dev)
    W1 = torch.from_numpy(datagen.normal((D, H), 71, 0.0, 1.0 / np.sqrt(D))).to(dev)
    W2 = torch.from_numpy(datagen.normal((H, H), 72, 0.0, 1.0 / np.sqrt(H))).to(dev)
    W2p = torch.from_numpy(datagen.normal((H, H), 73, 0.0, 1.0 / np.sqrt(H))).to(dev)
    W3 = torch.from_numpy(datagen.normal((H, D), 74, 0.0, 1.0 / np.sqrt(H))).to(dev)
    b1, b2, b3 = (torch.from_numpy(datagen.normal((n,), s, 0.0, 0.1)).to(dev) for n, s in ((H, 75), (H, 76), (D, 77)))
    h = torch.empty((Mx, H), device=dev)
    hw = torch.empty((Mx, H), device=dev)
    y = torch.empty((Mx, H), device=dev)
    o = torch.empty((Mx, D), device=dev)

    host = {k: v.cpu().numpy() for k, v in (("X", X), ("W1", W1), ("W2", W2), ("W2p", W2p), ("W3", W3),
                                             ("b1", b1), ("b2", b2), ("b3", b3))}

    def build_mlp(rg, r):
        # h = relu(X W1 + b1); y = relu(h W2 + b2) + h W2'; out = y W3 + b3 (rows of X independent)
        L = rg.lib
        w = {k: rg.input(v) for k, v in host.items() if k != "X"}
        hn = L.g_relu(L.g_add(L.g_matmul(rg.input(host["X"][:r]), w["W1"]), w["b1"]))
        yn = L.g_add(L.g_relu(L.g_add(L.g_matmul(hn, w["W2"]), w["b2"])), L.g_matmul(hn, w["W2p"]))
        return L.g_add(L.g_matmul(yn, w["W3"]), w["b3"])

    mlp_cpu = cpu_reference_ms(build_mlp, Mx, 2.0 * (D * H + 2 * H * H + H * D))
    del host

    def st(*items):
        arr = (mlib.EpStepDev * max(1, len(items)))()
        for i, it in enumerate(items):
            arr[i] = it
        return arr, len(items)

    s1 = st(mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, b1.data_ptr(), H, 0.0, 0), mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0))
    s2 = st(mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, b2.data_ptr(), H, 0.0, 0), mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0),
            mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, hw.data_ptr(), H, 0.0, 0))
    s3 = st(mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, b3.data_ptr(), D, 0.0, 0))
    for prec_name, prec in (("tf32", mlib.GPU_PRECISION_TF32), ("3xtf32", mlib.GPU_PRECISION_3XTF32)):
        def mlp():
            for a, lda, b, n, k, outp, (arr, ns) in (
                    (X, D, W1, H, D, h, s1), (h, H, W2p, H, H, hw, st()), (h, H, W2, H, H, y, s2), (y, H, W3, D, H, o, s3)):
                rc = lib.mxb_fused_gemm(ctx, a.data_ptr(), lda, b.data_ptr(), n, outp.data_ptr(), n, Mx, n, k, arr, ns,
                                        prec, stream.cuda_stream)
                assert rc == 0, mlib.last_error()
        tmin, tmed = time_launches(mlp, 10)
        flops = 2.0 * Mx * (D * H + 2 * H * H + H * D)
        line = {"sweep": "3-layer MLP DAG (4 GEMM launches)", "M": Mx, "D": D, "H": H, "precision": prec_name,
                "ms_min": tmin, "ms_median": tmed, "tflops": flops / (tmin * 1e-3) / 1e12}
        line.update(mlp_cpu)
        if mlp_cpu.get("cpu_reference_ms"):
            line["speedup_vs_cpu_reference"] = mlp_cpu["cpu_reference_ms"] / tmin
        print(json.dumps(line), flush=True)

        # The same DAG with h W2' fused into F2 (mxb_fused_gemm2): three launches.
        s2p = st(mlib.EpStepDev(mlib.MXB_EP_ADD_ROW, 0, b2.data_ptr(), H, 0.0, 0),
                 mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0),
                 mlib.EpStepDev(mlib.MXB_EP_ADD_PRODUCT, 0, None, 0, 0.0, 0))

        def mlp_fused():
            rc = lib.mxb_fused_gemm(ctx, X.data_ptr(), D, W1.data_ptr(), H, h.data_ptr(), H, Mx, H, D, s1[0], s1[1],
                                    prec, stream.cuda_stream)
            assert rc == 0, mlib.last_error()
            rc = lib.mxb_fused_gemm2(ctx, h.data_ptr(), H, W2.data_ptr(), H, h.data_ptr(), H, W2p.data_ptr(), H, H,
                                     y.data_ptr(), H, Mx, H, H, s2p[0], s2p[1], prec, stream.cuda_stream)
            assert rc == 0, mlib.last_error()
            rc = lib.mxb_fused_gemm(ctx, y.data_ptr(), H, W3.data_ptr(), D, o.data_ptr(), D, Mx, D, H, s3[0], s3[1],
                                    prec, stream.cuda_stream)
            assert rc == 0, mlib.last_error()
        tmin, tmed = time_launches(mlp_fused, 10)
        print(json.dumps({"sweep": "3-layer MLP DAG, h W2' fused into F2 (3 launches)", "M": Mx, "D": D, "H": H,
                          "precision": prec_name, "ms_min": tmin, "ms_median": tmed,
                          "tflops": flops / (tmin * 1e-3) / 1e12}), flush=True)
    lib.gpu_ctx_destroy(ctx)
    return 0


def run_kernels(args):
    """The library's HBM-bound kernels alone, operands larger than L2 (126 MB)
    and resident: standalone add (same shape: 12 B per element; [N] row
    broadcast: 8 B), relu (8 B), and the skinny GEMM, whose traffic is B
    (4*K*N bytes).  Each launch behind a ~50 us spin on the stream so the
    events bracket the kernel; min and median of 20.  Reported against the
    measured HBM copy rate."""
    import torch

    from minixla_b200 import lib as mlib

    lib = mlib.load()
    ctx = lib.gpu_ctx_create_on(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.Stream(dev)
    peak, peak_src = measured_hbm_gbs()

    def time_launches(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                torch.cuda._sleep(100_000)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return min(ts), statistics.median(ts)

    def report(name, nbytes, fn, extra=None):
        tmin, tmed = time_launches(fn)
        gbs = nbytes / (tmin * 1e-3) / 1e9
        line = {"kernel": name, "bytes": int(nbytes), "ms_min": tmin, "ms_median": tmed, "gbs": gbs,
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                             "peak_source": peak_src}}
        line.update(extra or {})
        print(json.dumps(line), flush=True)

    n = 64 << 20  # 64 Mi floats = 256 MiB per operand
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.rand(n, device=dev, generator=g) - 0.5
    b = torch.rand(n, device=dev, generator=g) - 0.5
    out = torch.empty(n, device=dev)
    row = torch.rand(8192, device=dev, generator=g)

    def add_same():
        assert lib.mxb_add(ctx, a.data_ptr(), n, b.data_ptr(), n, out.data_ptr(), stream.cuda_stream) == 0

    def add_row():
        assert lib.mxb_add(ctx, a.data_ptr(), n, row.data_ptr(), row.numel(), out.data_ptr(), stream.cuda_stream) == 0

    def relu():
        assert lib.mxb_relu(ctx, a.data_ptr(), n, out.data_ptr(), stream.cuda_stream) == 0

    report("add (same shape)", 12.0 * n, add_same, {"elements": n})
    torch.testing.assert_close(out, a + b)
    report("add ([8192] row broadcast)", 8.0 * n, add_row, {"elements": n})
    torch.testing.assert_close(out, a + row.repeat(n // 8192))
    report("relu", 8.0 * n, relu, {"elements": n})
    torch.testing.assert_close(out, torch.relu(a))
    del a, b, out

    # Skinny fused GEMM relu(x.B + c), M rows: the work is streaming B.
    K = N = 8192
    B = torch.rand(K, N, device=dev, generator=g) - 0.5
    for M in (1, 4, 16):
        x = torch.rand(M, K, device=dev, generator=g) - 0.5
        c = torch.rand(M, N, device=dev, generator=g) - 0.5
        y = torch.empty(M, N, device=dev)
        steps = (mlib.EpStepDev * 2)()
        steps[0] = mlib.EpStepDev(mlib.MXB_EP_ADD_FULL, 0, c.data_ptr(), N, 0.0, 0)
        steps[1] = mlib.EpStepDev(mlib.MXB_EP_RELU, 0, None, 0, 0.0, 0)

        def skinny():
            assert lib.mxb_fused_gemm(ctx, x.data_ptr(), K, B.data_ptr(), N, y.data_ptr(), N, M, N, K, steps, 2,
                                      mlib.GPU_PRECISION_TF32, stream.cuda_stream) == 0

        # Up to 8 rows the CUDA-core skinny kernel (fp32 products); from 9 the
        # TF32 tensor-core kernel with its K split.
        form = "CUDA-core fp32" if M <= 8 else "tensor-core TF32, K split"
        report(f"few-row fused GEMM M={M} ({form})", 4.0 * (K * N + M * K + 2 * M * N), skinny,
               {"M": M, "N": N, "K": K})
        ref = torch.relu(x.double() @ B.double() + c.double())
        assert float((y.double() - ref).norm() / ref.norm()) < (1e-5 if M <= 8 else 2e-3)
    lib.gpu_ctx_destroy(ctx)
    return 0


def run_mlp(args):
    """The 3-layer MLP through the reference-facing path (X 4096 x
    1024; W1 1024 x 4096, W2 and W2' 4096 x 4096, W3 4096 x 1024; bias rows)
    built with MiniXLA's own g_matmul / g_add / g_relu and optimize()
    (oracle/_ref), then handed to gpu_execute_into.  Each step is one
    synchronous call, host X in and host output out, timed on the host clock
    (the call returns with the result on the host).  Runs: weights uploaded
    every call (the reference's behaviour, gpu_exec.c:450-456) and kept
    resident (gpu_ctx_keep_resident); the row-streamed and the one-stream
    executors; both precision modes.  A few output rows are checked against
    the oracle."""
    import numpy as np
    import torch

    from minixla_b200 import datagen
    from minixla_b200 import lib as mlib
    from minixla_b200.abi import HostGraph
    from oracle.bindings import RefGraph, fused_oracle, ref_available

    if not ref_available():
        print(json.dumps({"workload": "3-layer MLP 4096x1024 -> 4096 -> 4096 -> 1024", "unavailable": "oracle/_ref not built"}))
        return 0
    lib = mlib.load()
    ctx = lib.gpu_ctx_create_on(0)
    Mx, D, H = 4096, 1024, 4096
    host = {
        "X": datagen.uniform((Mx, D), 70),
        "W1": datagen.normal((D, H), 71, 0.0, 1.0 / np.sqrt(D)),
        "W2": datagen.normal((H, H), 72, 0.0, 1.0 / np.sqrt(H)),
        "W2p": datagen.normal((H, H), 73, 0.0, 1.0 / np.sqrt(H)),
        "W3": datagen.normal((H, D), 74, 0.0, 1.0 / np.sqrt(H)),
        "b1": datagen.normal((H,), 75, 0.0, 0.1),
        "b2": datagen.normal((H,), 76, 0.0, 0.1),
        "b3": datagen.normal((D,), 77, 0.0, 0.1),
    }
    rg = RefGraph()
    L = rg.lib
    nodes = {k: rg.input(v) for k, v in host.items()}
    hn = L.g_relu(L.g_add(L.g_matmul(nodes["X"], nodes["W1"]), nodes["b1"]))
    yn = L.g_add(L.g_relu(L.g_add(L.g_matmul(hn, nodes["W2"]), nodes["b2"])), L.g_matmul(hn, nodes["W2p"]))
    root = rg.own(rg.optimize(L.g_add(L.g_matmul(yn, nodes["W3"]), nodes["b3"])))
    n_nodes = rg.node_count(root)
    out_h = torch.empty((Mx, D), dtype=torch.float32).pin_memory()
    hg = HostGraph()
    out_t = hg.tensor(out_h)
    flops = 2.0 * Mx * (D * H + 2 * H * H + H * D)

    rows = [0, 2047, 4095]
    X = host["X"][rows]
    h_ref = fused_oracle(X, host["W1"], [("add", host["b1"]), ("relu",)])
    hw_ref = fused_oracle(h_ref, host["W2p"], [])
    y_ref = fused_oracle(h_ref, host["W2"], [("add", host["b2"]), ("relu",), ("add", hw_ref)])
    want = fused_oracle(y_ref, host["W3"], [("add", host["b3"])])

    weights = ["W1", "W2", "W2p", "W3", "b1", "b2", "b3"]
    for prec_name, prec in (("tf32", mlib.GPU_PRECISION_TF32), ("3xtf32", mlib.GPU_PRECISION_3XTF32)):
        lib.gpu_ctx_set_precision(ctx, prec)
        for resident in (False, True):
            if resident:
                for k in weights:
                    assert lib.gpu_ctx_keep_resident(ctx, nodes[k].contents.output) == 0, mlib.last_error()
            for chunks in ("8", "1"):
                os.environ["MINIXLA_STREAM_CHUNKS"] = chunks
                for _ in range(2):
                    assert lib.gpu_execute_into(root, ctx, out_t) == 0, mlib.last_error()
                ts = []
                for _ in range(10):
                    t0 = time.perf_counter()
                    assert lib.gpu_execute_into(root, ctx, out_t) == 0, mlib.last_error()
                    ts.append(time.perf_counter() - t0)
                got = out_h.numpy()[rows]
                rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
                tol = 3 * (2e-3 if prec == mlib.GPU_PRECISION_TF32 else 1e-5)
                assert rel <= tol, f"MLP check failed: {rel:.3g} > {tol}"
                ms = min(ts) * 1e3
                h2d = 4 * Mx * D + (0 if resident else 4 * sum(host[k].size for k in weights))
                print(json.dumps({
                    "workload": "3-layer MLP 4096x1024 -> 4096 -> 4096 -> 1024 via optimize() + gpu_execute_into", "precision": prec_name,
                    "nodes_after_optimize": n_nodes, "weights": "resident" if resident else "uploaded each call",
                    "executor": "row-streamed (8 chunks)" if chunks == "8" else "one-stream (multi-stream DAG)",
                    "ms_min": ms, "ms_median": statistics.median(ts) * 1e3, "tflops": flops / (ms * 1e-3) / 1e12,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * Mx * D, "rel_err_rows": rel}), flush=True)
        lib.gpu_ctx_release_resident(ctx, None)
    os.environ.pop("MINIXLA_STREAM_CHUNKS", None)
    rg.close()
    lib.gpu_ctx_destroy(ctx)
    return 0


def run_batched(args):
    """A rank-3 fused node relu(A.B + C) -- `batch` products of M x N x K,
    eval_fused's batch loop (graph.c:80-113) -- timed kernel-only through
    gpu_time_kernel_ms: every product in one launch, and one launch per
    product (MINIXLA_BATCH_LAUNCH=0; that form's time includes the host's
    preparation of each launch, as a caller would see it).  Checked against
    the oracle on the first and last products."""
    import numpy as np

    from minixla_b200 import datagen
    from minixla_b200 import lib as mlib
    from minixla_b200.abi import OP_ADD, OP_RELU, HostGraph, free_host_tensor, tensor_to_numpy
    from oracle.bindings import fused_oracle

    bt, M, N, K = (int(v) for v in args.batched.split(","))
    lib = mlib.load()
    ctx = lib.gpu_ctx_create_on(0)
    A = datagen.uniform((bt, M, K), 0)
    B = datagen.uniform((bt, K, N), 1)
    Cm = datagen.normal((bt, M, N), 2)
    hg = HostGraph()
    root = hg.fused_node(hg.input_node(A), hg.input_node(B), [(OP_ADD, hg.input_node(Cm)), (OP_RELU, None)])
    flops = 2.0 * bt * M * N * K
    for prec_name, prec in (("tf32", mlib.GPU_PRECISION_TF32), ("3xtf32", mlib.GPU_PRECISION_3XTF32)):
        lib.gpu_ctx_set_precision(ctx, prec)
        t = lib.gpu_execute(root, ctx)
        if not t:
            raise RuntimeError(mlib.last_error())
        got = tensor_to_numpy(t)
        free_host_tensor(t)
        err = 0.0
        for b in (0, bt - 1):
            want = fused_oracle(A[b], B[b], [("add", Cm[b]), ("relu",)])
            err = max(err, float(np.linalg.norm(got[b] - want) / np.linalg.norm(want)))
        line = {"batched": "fused relu(A.B+C), rank 3", "batch": bt, "M": M, "N": N, "K": K,
                "precision": prec_name, "rel_err_first_last": err}
        for form, env in (("one_launch", "1"), ("launch_per_product", "0")):
            os.environ["MINIXLA_BATCH_LAUNCH"] = env
            ms = lib.gpu_time_kernel_ms(root, ctx, 3, 10)
            if ms <= 0:
                raise RuntimeError(mlib.last_error())
            line[form] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12}
        os.environ.pop("MINIXLA_BATCH_LAUNCH", None)
        print(json.dumps(line), flush=True)
    lib.gpu_ctx_destroy(ctx)
    return 0


def main():
    args = parse()
    rank, local_rank, world = env_rank()
    if args.batched:
        return run_batched(args)
    if args.sweep:
        return run_sweep(args)
    if args.kernels:
        return run_kernels(args)
    if args.mlp:
        return run_mlp(args)
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    return ours_arm(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
