"""Host side of a sharded decode step whose kernel gathers the outputs itself.

One process per GPU. Every rank allocates its global output buffers (``nbuf`` of them, used in turn
by consecutive steps) and a signal array in CUDA IPC memory (``kvb_ipc_alloc``); the 64-byte handles
go to every rank over ``torch.distributed`` (``all_gather_object``), and each rank maps the others'
memory (``kvb_ipc_open``). A step is then two launches on the rank's stream:
``kvb_paged_decode_gather_async``, whose kernel writes each finished output row into every rank's
buffer at its global position, and ``kvb_peer_barrier_async``, after which this rank's buffer holds
the whole step. No NCCL call and no reorder are left in the step.

Two buffers suffice for a consumer on the rank's own stream: step i + 2 writes buffer i % 2 on a
peer only after that peer passed the barrier of step i + 1, which its stream reaches after whatever
it ran on step i's output.
"""
from __future__ import annotations

from typing import List, Optional

import kv_cache_bench_b200 as kvb


class _DeviceArray:
    """A device pointer seen through __cuda_array_interface__ (torch.as_tensor wraps it without a
    copy and without taking ownership)."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3}


class PeerGather:
    """Buffers, mappings and launch arguments of the in-kernel gather on this rank.

    rows, heads, head_dim: the global output [rows][heads][head_dim] (fp32). out_head0: the global
    head of this rank's head 0 (KV-head shards). out_rows: int32 device tensor, the global row of
    each local sequence (sequence shards), or None when local sequence b is global row b."""

    def __init__(self, torch, dist, rank: int, world: int, rows: int, heads: int, head_dim: int, device,
                 out_head0: int = 0, out_rows=None, nbuf: int = 2, timeout_us: int = 0):
        if not 1 <= world <= kvb.MAX_PEERS:
            raise ValueError(f"the in-kernel gather serves 1..{kvb.MAX_PEERS} ranks")
        self.torch, self.dist, self.rank, self.world, self.nbuf = torch, dist, rank, world, nbuf
        self._own: List[int] = []
        self._opened: List[int] = []
        nbytes = rows * heads * head_dim * 4
        mine, handles = [], []
        for _ in range(nbuf):
            p, h = kvb.ipc_alloc(nbytes)
            self._own.append(p)
            mine.append(p)
            handles.append(h)
        sig, h = kvb.ipc_alloc(4 * kvb.MAX_PEERS)
        self._own.append(sig)
        handles.append(h)
        every: List[Optional[list]] = [None] * world
        dist.all_gather_object(every, handles)
        self.buffers = [[0] * world for _ in range(nbuf)]
        self.signals = [0] * world
        for j in range(world):
            for b in range(nbuf):
                self.buffers[b][j] = mine[b] if j == rank else self._open(every[j][b])
            self.signals[j] = sig if j == rank else self._open(every[j][nbuf])
        self.epoch = torch.zeros(4, dtype=torch.int32, device=device)  # word 0: this rank's step count
        self.out_rows = out_rows
        rows_ptr = out_rows.data_ptr() if out_rows is not None else 0
        self.args = [kvb.peer_out(self.buffers[b], rank, rows, heads, out_head0, rows_ptr) for b in range(nbuf)]
        self.barrier = kvb.peer_barrier_args(rank, self.signals, self.epoch.data_ptr(), timeout_us)
        self._mine, self._shape, self._device, self._views = mine, (rows, heads, head_dim), device, None
        torch.cuda.synchronize()  # the epoch word is zero before any barrier kernel reads it
        dist.barrier()

    @property
    def views(self):
        """This rank's global output buffers as torch tensors (no copy, not owned)."""
        if self._views is None:
            self._views = [self.torch.as_tensor(_DeviceArray(p, self._shape), device=self._device) for p in self._mine]
        return self._views

    def _open(self, handle: bytes) -> int:
        p = kvb.ipc_open(handle)
        self._opened.append(p)
        return p

    def launch(self, cargs, workspace: int, workspace_bytes: int, stream: int, i: int):
        """Step i: the decode with the in-kernel gather, then the step barrier. Returns this rank's
        global output of the step (valid on `stream` after the barrier)."""
        b = i % self.nbuf
        kvb.paged_decode_gather_async(cargs, self.args[b], workspace, workspace_bytes, stream)
        kvb.peer_barrier_async(self.barrier, workspace, stream)
        return self.views[b]

    def close(self) -> None:
        """Unmaps the peers' memory and frees this rank's, once every rank is done with it."""
        if not self._own:
            return
        self.torch.cuda.synchronize()
        self.dist.barrier()
        for p in self._opened:
            kvb.ipc_close(p)
        self._opened = []
        self.dist.barrier()
        self._views, self._mine = None, []
        for p in self._own:
            kvb.ipc_free(p)
        self._own = []
