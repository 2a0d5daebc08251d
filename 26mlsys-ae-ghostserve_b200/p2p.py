"""Peer mapping of KV shard buffers across the ranks of one node (CUDA IPC).

The reference moves every rank's delta KV to one destination rank with two
NCCL gathers per hook call (bench_ghostserve_rdp.py:303-332) and then packs
and encodes there.  Here each rank exports its shard buffers once (a 64-byte
CUDA IPC handle + offset per buffer), the handles go around the process group
(``all_gather_object`` — control plane only), and every rank maps its peers'
buffers.  The encode kernel then reads peer shards in place with NVLink peer
loads; no copy kernel or NCCL data call sits on that path.

Peer memory is read by plain per-CTA cp.async.bulk copies (each CTA loads
its own copy into its own shared memory; no cluster multicast anywhere), or by
16-byte loads.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, List, Optional, Sequence

import torch
import torch.distributed as dist

from . import _lib


def _export(t: torch.Tensor):
    handle = (C.c_char * _lib.IPC_HANDLE_BYTES)()
    off = C.c_int64(0)
    _lib.call("gsec_ipc_export", C.c_void_p(t.data_ptr()), C.cast(handle, C.c_void_p), C.byref(off))
    return bytes(handle), int(off.value)


def _import(handle: bytes, offset: int) -> int:
    buf = C.create_string_buffer(handle, _lib.IPC_HANDLE_BYTES)
    out = C.c_void_p(0)
    _lib.call("gsec_ipc_import", C.cast(buf, C.c_void_p), int(offset), C.byref(out))
    return int(out.value)


class PeerGroup:
    """ptr(r, j) is the address, valid on this rank's GPU, of buffer j of rank r."""

    def __init__(self, table: List[List[int]], rank: int, world: int, keep: Sequence[torch.Tensor],
                 closer: Optional[Callable[[], None]]):
        self.table = table
        self.rank = rank
        self.world = world
        self._keep = list(keep)
        self._closer = closer

    @classmethod
    def create(cls, buffers: Sequence[torch.Tensor], group=None, exporter=_export, importer=_import,
               closer=None) -> "PeerGroup":
        """Collective: every rank passes the same number of buffers."""
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        mine = [exporter(t) + (t.numel() * t.element_size(),) for t in buffers]
        everyone: List = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        if any(len(e) != len(mine) for e in everyone):
            raise ValueError("every rank must share the same number of buffers")
        table = []
        for r in range(world):
            if r == rank:
                table.append([t.data_ptr() for t in buffers])
            else:
                table.append([importer(h, off) for (h, off, _n) in everyone[r]])
        if closer is None and importer is _import:
            def closer():
                _lib.call("gsec_ipc_close_all")
        return cls(table, rank, world, buffers, closer)

    def ptr(self, r: int, j: int) -> int:
        return self.table[r][j]

    def close(self) -> None:
        """Unmap peer buffers. Call after a barrier that follows the last kernel
        reading them."""
        if self._closer is not None:
            self._closer()
            self._closer = None
        self.table = []


def codeword_placement(rank: int, world: int, k: int) -> List[int]:
    """Ranks holding data shards 0..k-1 of the codeword owned by ``rank``:
    shard j sits on (rank + j) mod world, so shard 0 is local and the other
    shards spread over the peers."""
    return [(rank + j) % world for j in range(k)]


def stripe_slice(rank: int, world: int, nstripes: int):
    """Contiguous share [lo, hi) of nstripes for rank (sizes differ by <= 1)."""
    base, extra = divmod(nstripes, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)
