"""Row all-gather written by the fused GEMM itself, for one process per GPU.

Rank r of a row-sharded job owns rows [r0, r1) of out = epi(A @ B)
(``mxb_shard_rows``).  A consumer that needs the whole [M, N] tensor on every
GPU would run an NCCL all-gather after the kernels; ``GatherBuffers`` instead
gives every rank a full-size output buffer that all ranks can write (CUDA IPC
mappings exchanged over ``torch.distributed``), and ``GatherBuffers.gemm``
calls ``mxb_fused_gemm_allgather``, whose epilogue writes this rank's rows
into its own buffer and into every peer's over NVLink.

Peer rows are complete once the writing rank's kernel has finished, so a
reader synchronises the ranks first: ``GatherBuffers.barrier`` (a one-element
all-reduce on the given stream) does that.  ``close`` unmaps the peers'
buffers, waits for every rank to do the same and frees the local one.

``lib`` is the loaded native library (``minixla_b200.lib.load()``); the
``torch.distributed`` process group must be initialised.
"""
from __future__ import annotations

import ctypes as C

from .lib import MXB_IPC_HANDLE_BYTES, MXB_MAX_PEERS, last_error


class _DeviceArray:
    """A raw device allocation seen through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape: tuple, strides_bytes: tuple):
        self.__cuda_array_interface__ = {
            "shape": shape, "typestr": "<f4", "data": (ptr, False), "version": 3, "strides": strides_bytes,
        }


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {last_error()}")


class GatherBuffers:
    """Every rank's [rows_total, cols] fp32 output (row pitch ``ldo``),
    mapped into this process; ``peer_rows(row0)`` are the addresses of row
    ``row0`` in the other ranks' copies, in ``peer_order()``."""

    def __init__(self, lib, device: int, rows_total: int, cols: int, ldo: int | None = None, group=None):
        import torch.distributed as dist

        self.lib, self.device, self.group = lib, device, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world - 1 > MXB_MAX_PEERS:
            raise ValueError(f"at most {MXB_MAX_PEERS + 1} ranks share one row all-gather")
        self.rows_total, self.cols = rows_total, cols
        self.ldo = ldo if ldo is not None else cols
        if self.ldo < cols:
            raise ValueError("ldo < cols")
        nbytes = 4 * rows_total * self.ldo
        ptr = C.c_void_p()
        handle = (C.c_ubyte * MXB_IPC_HANDLE_BYTES)()
        _check(lib.mxb_ipc_alloc(device, nbytes, C.byref(ptr), handle), "mxb_ipc_alloc")
        self.local = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.remote = {}  # rank -> base address of that rank's buffer in this process
        try:
            for r, h in enumerate(handles):
                if r == self.rank:
                    continue
                p = C.c_void_p()
                buf = (C.c_ubyte * MXB_IPC_HANDLE_BYTES).from_buffer_copy(h)
                _check(lib.mxb_ipc_open(device, buf, C.byref(p)), "mxb_ipc_open")
                self.remote[r] = p.value
        except Exception:
            self._unmap()
            raise

    def tensor(self):
        """This rank's full buffer as a torch tensor (no copy)."""
        import torch

        arr = _DeviceArray(self.local, (self.rows_total, self.cols), (4 * self.ldo, 4))
        return torch.as_tensor(arr, device=torch.device("cuda", self.device))

    def local_rows(self, row0: int) -> int:
        return self.local + 4 * row0 * self.ldo

    def peer_order(self):
        """The other ranks, starting after this one (rank + 1, rank + 2, ...,
        wrapping): every rank lists a different peer first, so the ranks'
        kernels do not all store to the same GPU at the same time."""
        return [(self.rank + i) % self.world for i in range(1, self.world)]

    def peer_rows(self, row0: int):
        ptrs = [self.remote[r] + 4 * row0 * self.ldo for r in self.peer_order()]
        return (C.c_void_p * max(1, len(ptrs)))(*ptrs), len(ptrs)

    def gemm(self, ctx, A: int, lda: int, B: int, ldb: int, row0: int, M: int, N: int, K: int, steps, n_steps: int,
             precision: int, stream: int) -> int:
        """Rows row0 .. row0 + M of epi(A @ B) into every rank's buffer
        (``mxb_fused_gemm_allgather``); returns its status code."""
        if N != self.cols or row0 < 0 or row0 + M > self.rows_total:
            raise ValueError("rows or columns outside the gather buffer")
        peers, n = self.peer_rows(row0)
        return self.lib.mxb_fused_gemm_allgather(ctx, A, lda, B, ldb, self.local_rows(row0), self.ldo, peers, n, M, N,
                                                 K, steps, n_steps, precision, stream)

    def barrier(self, stream=None) -> None:
        """Orders every rank's earlier work on its stream before later work
        on this rank's stream (a one-element all-reduce)."""
        import torch
        import torch.distributed as dist

        ctx = torch.cuda.stream(stream) if stream is not None else torch.cuda.stream(torch.cuda.current_stream())
        with ctx:
            flag = torch.zeros(1, device=torch.device("cuda", self.device))
            dist.all_reduce(flag, group=self.group)

    def _unmap(self) -> None:
        for r in list(self.remote):
            self.lib.mxb_ipc_close(self.device, self.remote.pop(r))

    def close(self) -> None:
        import torch.distributed as dist

        if self.local is None:
            return
        self._unmap()
        dist.barrier(group=self.group)  # no rank still maps this buffer
        self.lib.mxb_ipc_free(self.device, self.local)
        self.local = None
