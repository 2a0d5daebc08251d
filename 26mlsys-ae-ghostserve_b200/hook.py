"""Drop-in for the reference's KV fault-tolerance hook on SGLang's FlashInfer
backend (bench_ghostserve_rdp.py:212-532).

``patch_backend(backend, ft)`` replaces ``backend.forward_extend`` exactly like
``_patch_flashinfer_backend`` (:396-481): the wrapper forwards every argument,
always returns the original result and swallows (and logs) any error of the
fault-tolerance work.  After each extend call, ``ft.on_extend`` takes the
prefill-delta KV (``kv_pool[slot_mapping != -1]``, :440-458) and protects it:

mode="reference"  the reference flow, bit for bit: chunk id from rank 0
                  (:287-301), NCCL gather of every rank's K and V to the
                  rotating destination rank (:303-332), fp16 value cast, pack,
                  mod-S row/diagonal parity and a copy of P and Q to the host
                  (:334-392) — with libgsec's kernels instead of the JIT ones.
mode="fused"      the B200 path: every rank gathers its delta KV out of the
                  pool through the slot list (one kernel per plane, a -1 slot is
                  a zero row) into a buffer the other ranks have mapped (CUDA
                  IPC); after one stream-ordered barrier each rank encodes its
                  1/world slice of the stripes, reading all ranks' KV with NVLink
                  peer loads inside the encode kernel, and offloads its parity
                  slice to pinned host memory asynchronously, where it stays
                  for recover_pool / recover_parts.  No NCCL data gather, no
                  value cast (raw KV bytes), no host sync.

Both modes append the reference's JSONL record (:377-389) to FT_METRICS_FILE.
"""
from __future__ import annotations

import functools
import json
import os
import time
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib, codec, ext
from .store import ParityStore

ENV_FLAG = "SGLANG_GATHER_KV_TO_GPU0"
LOG_PREFIX = "[ft-rdp]"


def _log(msg: str) -> None:
    try:
        print(f"{LOG_PREFIX} {msg}", flush=True)
    except Exception:
        pass


@dataclass
class HookConfig:
    mode: str = "fused"                 # "fused" | "reference"
    scheme: str = "rdp"                 # fused mode code: "rdp" | "xor" | "rs8"
    rs_parity: int = 2
    unit: int = 4096                    # RDP stripe unit
    star_base: int = field(default_factory=lambda: int(os.getenv("RDP_STAR_BASE", "0")))
    metrics_file: Optional[str] = field(default_factory=lambda: os.getenv("FT_METRICS_FILE"))
    prog_start_mono: float = field(default_factory=lambda: float(os.getenv("FT_PROG_START_MONO", "nan")))
    compat_cast_fp16: bool = True       # reference mode: .to(float16) as bench_ghostserve_rdp.py:345-346
    broadcast_chunk_id: bool = True     # reference mode: rank-0 counter + broadcast (:287-301)
    protect: str = "call"               # fused mode: "call" encodes after every forward_extend call (as the
                                        # reference does); "chunk" encodes once per prefill chunk, after the
                                        # chunk_layers-th call, all layers' delta KV in one codeword
    chunk_layers: int = field(default_factory=lambda: int(os.getenv("FT_CHUNK_LAYERS", "0")))
    offload: bool = True                # copy parity to pinned host memory
    host_keep: int = 256                # chunks whose parity slice stays in pinned host memory
    host_budget: int = 1 << 30          # bytes of the pinned ring holding them (at least 4 chunks' worth)
    verbose: bool = False


class KVFaultTolerance:
    """Per-process state of the hook (the module globals of the reference plugin)."""

    def __init__(self, config: Optional[HookConfig] = None, group=None):
        self.cfg = config or HookConfig()
        self.group = group
        self.chunk_counter = 0
        self.first_chunk_wall_ms = None
        self.records = []
        self._staging = None      # fused mode: registered KV staging (2 slots)
        self._peers = None
        self._parity = None
        # chunk id -> this rank's parity slice in pinned host memory
        self._store = ParityStore(self.cfg.host_keep, self.cfg.host_budget, pin=True,
                                  before_release=self._copies_landed)
        self._pending = []        # (record, event, t_enqueue) awaiting D2H completion
        self._copy_stream = None
        self._parity_free = [None, None]
        self._calls = 0
        self._bar_t = None        # the barrier's all-reduce operand
        self._plans = {}          # (slot, half, stream) -> marshalled encode of that staging slot
        self._pools = {}          # KV pool geometry by (pointer, shape, strides)
        self._events = []         # timing events free for reuse
        self._chunk_pools = []    # protect="chunk": this chunk's pools seen so far (one per layer call)

    # ------------------------------------------------------------- control --
    def _rank_world(self):
        return dist.get_rank(self.group), dist.get_world_size(self.group)

    def next_chunk_id(self, device=None):
        """(chunk_id, dst_rank) with dst = (chunk_id - 1) % world (:287-301)."""
        rank, world = self._rank_world()
        if self.cfg.mode == "reference" and self.cfg.broadcast_chunk_id:
            if rank == 0:
                self.chunk_counter += 1
            t = torch.tensor([self.chunk_counter], device=device, dtype=torch.int64)
            dist.broadcast(t, src=dist.get_global_rank(self.group, 0) if self.group else 0, group=self.group)
            cid = int(t.item())
            self.chunk_counter = cid
        else:
            # every rank runs the hook once per extend call, so a local counter
            # gives the same id everywhere without a broadcast or a host sync
            self.chunk_counter += 1
            cid = self.chunk_counter
        return cid, (cid - 1) % world

    def _barrier(self, device):
        """Stream-ordered on NCCL (a 1-element all-reduce); host-side otherwise."""
        if dist.get_backend(self.group) == "nccl":
            if self._bar_t is None or self._bar_t.device != torch.device(device):
                self._bar_t = torch.zeros(1, device=device)
            dist.all_reduce(self._bar_t, group=self.group)
        else:
            torch.cuda.current_stream(device).synchronize()
            dist.barrier(group=self.group)

    # ---------------------------------------------------- reference flow ----
    def gather_kv(self, local_k, local_v, dst_rank):
        """_distributed_gather_kv, bench_ghostserve_rdp.py:303-332."""
        rank, world = self._rank_world()
        kf = local_k.contiguous().view(-1)
        vf = local_v.contiguous().view(-1)
        elems = int(kf.numel())
        if elems == 0:
            return None
        dst = dist.get_global_rank(self.group, dst_rank) if self.group else dst_rank
        if rank == dst_rank:
            k_all = torch.empty(elems * world, dtype=kf.dtype, device=kf.device)
            v_all = torch.empty(elems * world, dtype=vf.dtype, device=vf.device)
            dist.gather(kf, gather_list=[k_all.narrow(0, i * elems, elems) for i in range(world)], dst=dst,
                        group=self.group)
            dist.gather(vf, gather_list=[v_all.narrow(0, i * elems, elems) for i in range(world)], dst=dst,
                        group=self.group)
            return k_all, v_all, elems
        dist.gather(kf, gather_list=None, dst=dst, group=self.group)
        dist.gather(vf, gather_list=None, dst=dst, group=self.group)
        return None

    def compute_parity_to_cpu(self, K_all, V_all, elems, chunk_id, dst_rank):
        """_compute_parity_to_cpu, bench_ghostserve_rdp.py:334-392, on libgsec."""
        world = int(K_all.numel() // elems)
        S = 2 * elems
        rows = torch.empty((world + 2, S), dtype=torch.uint16, device=K_all.device)
        for r in range(world):
            k = K_all.narrow(0, r * elems, elems)
            v = V_all.narrow(0, r * elems, elems)
            if self.cfg.compat_cast_fp16:
                k, v = k.to(torch.float16), v.to(torch.float16)
            ext.rdp_kv_ops.pack_row_from_block(k.view(1, 1, elems, 1), v.view(1, 1, elems, 1), rows, r)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        ext.rdp_kv_ops.compute_rdp_parity(rows, nd=world, S=S, star_base=self.cfg.star_base)
        e1.record()
        torch.cuda.synchronize()
        encode_ms = float(e0.elapsed_time(e1))
        t0 = time.perf_counter()
        P_cpu = rows[world].to("cpu", non_blocking=True).contiguous()
        Q_cpu = rows[world + 1].to("cpu", non_blocking=True).contiguous()
        torch.cuda.synchronize()
        d2h_ms = (time.perf_counter() - t0) * 1000.0
        t1 = time.perf_counter()
        _ = P_cpu.to(rows.device, non_blocking=True)
        _ = Q_cpu.to(rows.device, non_blocking=True)
        torch.cuda.synchronize()
        h2d_ms = (time.perf_counter() - t1) * 1000.0
        rec = self._record(chunk_id, dst_rank, encode_ms, d2h_ms, h2d_ms, int((P_cpu.numel() + Q_cpu.numel()) * 2))
        self._emit(rec)
        return P_cpu, Q_cpu

    # -------------------------------------------------------- fused flow ----
    def _spec(self, world: int) -> codec.CodeSpec:
        if self.cfg.scheme == "xor":
            return codec.CodeSpec.xor(world)
        if self.cfg.scheme == "rs8":
            return codec.CodeSpec.rs8(world, self.cfg.rs_parity)
        return codec.CodeSpec.rdp(world, unit=self.cfg.unit)

    def _ensure_staging(self, nbytes_half: int, device):
        from . import p2p

        rank, world = self._rank_world()
        if self._staging is not None and self._staging[0][0].numel() >= nbytes_half:
            return
        if self._peers is not None:
            self._barrier(device)
            torch.cuda.synchronize(device)
            self._peers.close()
        cap = max(nbytes_half, 1 << 20)
        cap = -(-cap // 4096) * 4096
        # two slots, each a K buffer and a V buffer; peers read them in place
        self._staging = [[torch.empty(cap, dtype=torch.uint8, device=device) for _ in range(2)] for _ in range(2)]
        self._plans.clear()
        flat = [t for slot in self._staging for t in slot]
        self._peers = p2p.PeerGroup.create(flat, group=self.group)

    def _stage(self, slot, half, parts_k, parts_v):
        """Copy a shard's K parts then V parts into staging slot `slot`."""
        for parts, buf in ((parts_k, self._staging[slot][0]), (parts_v, self._staging[slot][1])):
            if all(t.is_contiguous() for t in parts):
                torch.cat([t.reshape(-1).view(torch.uint8) for t in parts], out=buf[:half])
            else:  # strided views: one copy each, straight into the staging buffer
                off = 0
                for t in parts:
                    n = t.numel() * t.element_size()
                    buf[off:off + n].view(t.dtype).view(t.shape).copy_(t)
                    off += n

    def _unstage(self, slot, parts_k, parts_v):
        """Inverse of _stage: scatter staging slot `slot` back into the parts."""
        for parts, buf in ((parts_k, self._staging[slot][0]), (parts_v, self._staging[slot][1])):
            off = 0
            for t in parts:
                n = t.numel() * t.element_size()
                t.copy_(buf[off:off + n].view(t.dtype).view(t.shape))
                off += n

    def recover_parts(self, chunk_id: int, lost, parts_k, parts_v):
        """Rebuild the KV shard of chunk `chunk_id` on the lost ranks (at most m).

        Collective over the group, replacement ranks included. Surviving ranks
        pass their chunk's K and V parts (as at encode time) and re-stage them;
        every rank copies its parity slice of the chunk from the host store back
        to the device and decodes its stripe slice, reading the survivors'
        staging with NVLink peer loads and writing the rebuilt stripes straight
        into the lost ranks' staging buffers; the lost ranks then scatter their
        staging into `parts_k` / `parts_v`. The host parity store is assumed to
        outlive a lost GPU (node memory); a parity slice is only recoverable while
        its chunk is still in the store."""
        half = sum(t.numel() * t.element_size() for t in parts_k)
        self._recover_staged(chunk_id, lost, half, parts_k[0].device,
                             lambda slot: self._stage(slot, half, parts_k, parts_v),
                             lambda slot: self._unstage(slot, parts_k, parts_v))

    def recover_pool(self, chunk_id: int, lost, kv_pool, slots: torch.Tensor):
        """recover_parts for a chunk encoded by encode_pool (one pool) or
        encode_pools (a list of per-layer pools, the hook's per-chunk mode):
        survivors gather the slot list's rows again, the lost ranks' rebuilt rows
        are scattered back into their pools at the same slots (rows of negative
        slots untouched)."""
        pools = list(kv_pool) if isinstance(kv_pool, (list, tuple)) else [kv_pool]
        geo = self._pools_geometry(pools)
        half = len(pools) * slots.numel() * geo[0]
        self._recover_staged(chunk_id, lost, half, pools[0].device,
                             lambda slot: self._gather_pools(pools, geo, slots, slot, True),
                             lambda slot: self._gather_pools(pools, geo, slots, slot, False))

    def _recover_staged(self, chunk_id, lost, half, device, stage, unstage):
        rank, world = self._rank_world()
        lost = sorted(set(int(r) for r in lost))
        if not lost:
            return
        entry = self._store.get(chunk_id)
        if entry is None:
            raise KeyError(f"parity of chunk {chunk_id} is no longer in the host store")
        spec, lo, hi = entry["spec"], entry["lo"], entry["hi"]
        if len(lost) > spec.m:
            raise ValueError(f"{len(lost)} lost ranks exceed the code's {spec.m} parity shards")
        if half != entry["half"]:
            raise ValueError("the chunk's KV does not match the encoded chunk size")
        slot = self._calls % 2
        self._calls += 1
        if rank not in lost:
            stage(slot)
        if hi > lo:
            par = self._parity_bufs(hi - lo, spec.m, device)[slot]
            if self._parity_free[slot] is not None:
                torch.cuda.current_stream(device).wait_event(self._parity_free[slot])
            torch.cuda.current_stream(device).wait_event(entry["copied"])
            n = hi - lo
            for j in range(spec.m):
                par[j][:n].copy_(entry["host"][j * n:(j + 1) * n], non_blocking=True)
        self._barrier(device)  # survivors' staging written; every parity slice on its device
        if hi > lo:
            shard_lo = [self._peers.ptr(r, 2 * slot) for r in range(world)] + [t.data_ptr() - lo for t in par]
            shard_hi = [self._peers.ptr(r, 2 * slot + 1) for r in range(world)] + [None] * spec.m
            codec.decode_ptrs(spec, shard_lo, shard_hi, half, 2 * half, lost, lo, hi)
        self._barrier(device)  # every slice of the lost shards has landed
        if rank in lost:
            unstage(slot)

    def encode_chunk(self, local_k: torch.Tensor, local_v: torch.Tensor, chunk_id: int):
        """Fused P2P encode of this rank's slice; returns the device parity slices."""
        return self.encode_parts([local_k], [local_v], chunk_id)

    def encode_parts(self, parts_k, parts_v, chunk_id: int):
        """Like encode_chunk for a shard made of several tensors (e.g. one chunk's
        K and V in every layer of a layer-major cache): the parts are copied once,
        in order, into this rank's peer-mapped staging buffer (K parts, then V
        parts), and the fused encode reads every rank's staging in place."""
        device = parts_k[0].device
        half = sum(t.numel() * t.element_size() for t in parts_k)
        if half % 16 or sum(t.numel() * t.element_size() for t in parts_v) != half:
            raise ValueError("delta K and V must have equal sizes, multiples of 16 bytes")
        self._ensure_staging(half, device)
        slot = self._calls % 2
        self._calls += 1
        self._stage(slot, half, parts_k, parts_v)
        return self._encode_staged(slot, half, chunk_id, device)

    def encode_pool(self, kv_pool: torch.Tensor, slots: torch.Tensor, chunk_id: int):
        """encode_chunk of one extend call's delta KV read straight out of the KV
        pool [slots, 2 (K, V), heads, head_dim] through its slot list: one
        gather kernel writes the K rows and the V rows into the staging buffer
        (a negative slot is a zero row), so neither the active count nor the
        gathered K/V ever reaches the host (bench_ghostserve_rdp.py:449-458 reads
        the count back and copies the rows twice). Every rank of the group must
        pass a slot list of the same length (tensor-parallel ranks share it)."""
        return self.encode_pools([kv_pool], slots, chunk_id)

    def encode_pools(self, pools, slots: torch.Tensor, chunk_id: int):
        """encode_pool over several pools that share one slot list (the
        per-layer pools of one prefill chunk): one gather launch stages every
        layer's K and V rows ([pool 0 K, pool 0 V, pool 1 K, ...]), then one
        barrier, one sliced encode and one host copy protect the whole chunk."""
        pools = list(pools)
        device = pools[0].device
        geo = self._pools_geometry(pools)
        half = len(pools) * slots.numel() * geo[0]
        if half % 16:
            raise ValueError("pool rows must be multiples of 16 bytes")
        self._ensure_staging(half, device)
        slot = self._calls % 2
        self._calls += 1
        self._gather_pools(pools, geo, slots, slot, True)
        return self._encode_staged(slot, half, chunk_id, device)

    def _pool_geometry(self, kv_pool):
        """(row bytes, slot pitch, V plane offset) of the pool, checked once per pool."""
        key = (kv_pool.data_ptr(), tuple(kv_pool.shape), tuple(kv_pool.stride()), kv_pool.dtype)
        geo = self._pools.get(key)
        if geo is None:
            row, pitch, _ = codec._pool_geometry(kv_pool, 0)
            _, _, voff = codec._pool_geometry(kv_pool, 1)
            geo = self._pools[key] = (row, pitch, voff)
        return geo

    def _pools_geometry(self, pools):
        """The common geometry of a list of pools (every pool checked, cached)."""
        geo = self._pool_geometry(pools[0])
        rows = pools[0].shape[0]
        for p in pools[1:]:
            if self._pool_geometry(p) != geo or p.shape[0] != rows or p.device != pools[0].device:
                raise ValueError("the pools of one chunk must share shape, strides, dtype and device")
        return geo

    def _gather_pools(self, pools, geo, slots, slot, gather: bool):
        """K and V planes of the slot list's rows in every pool into (gather) or
        out of (scatter) staging slot `slot`: one gsec_slots_*_pools call; the
        row stream [pool 0 K, pool 0 V, pool 1 K, ...] runs through the K
        buffer and on into the V buffer."""
        if slots.dtype not in (torch.int32, torch.int64) or not slots.is_contiguous() or \
                slots.device != pools[0].device:
            raise ValueError("slots must be a contiguous int32/int64 tensor on the pool's device")
        row, pitch, voff = geo
        fn = _lib.lib().gsec_slots_gather_pools if gather else _lib.lib().gsec_slots_scatter_pools
        n = slots.numel()
        half = len(pools) * n * row
        stream = torch.cuda.current_stream(pools[0].device).cuda_stream
        ptrs = _lib.ptr_array([p.data_ptr() for p in pools])
        _lib.check(fn(ptrs, len(pools), pitch, voff, 2, row, slots.data_ptr(), slots.element_size(), n,
                      pools[0].shape[0], self._staging[slot][0].data_ptr(), self._staging[slot][1].data_ptr(), half,
                      stream))

    def _parity_bufs(self, nbytes: int, m: int, device):
        """The two device parity slots (m buffers each) with room for nbytes."""
        if self._parity is None or len(self._parity[0]) != m or self._parity[0][0].numel() < max(nbytes, 16):
            if self._parity is not None:
                for ev in self._parity_free:  # host copies still reading the old buffers
                    if ev is not None:
                        ev.synchronize()
            self._parity = [[torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device) for _ in range(m)]
                            for _ in range(2)]
            self._parity_free = [None, None]
            self._plans.clear()
        return self._parity

    def _plan(self, slot: int, half: int, device):
        """Stripe slice, parity views and the marshalled encode of staging slot
        `slot` holding half-byte K and V halves (built once per shape)."""
        from . import p2p

        stream = torch.cuda.current_stream(device).cuda_stream
        key = (slot, half, stream)
        plan = self._plans.get(key)
        if plan is None:
            rank, world = self._rank_world()
            spec = self._spec(world)
            data_bytes = 2 * half
            g = spec.stripe_bytes()
            lo, hi = p2p.stripe_slice(rank, world, spec.parity_bytes(data_bytes) // g)
            lo, hi = lo * g, hi * g
            parity = self._parity_bufs(hi - lo, spec.m, device)[slot]
            enc = None
            if hi > lo:
                enc = codec.PreparedEncode(spec, [self._peers.ptr(r, 2 * slot) for r in range(world)],
                                           [self._peers.ptr(r, 2 * slot + 1) for r in range(world)], half,
                                           data_bytes, [t.data_ptr() - lo for t in parity], lo, hi, stream)
            plan = self._plans[key] = dict(spec=spec, lo=lo, hi=hi, enc=enc, views=[t[:hi - lo] for t in parity])
        return plan

    def _event(self):
        return self._events.pop() if self._events else torch.cuda.Event(enable_timing=True)

    def _encode_staged(self, slot: int, half: int, chunk_id: int, device):
        """Encode this rank's stripe slice of the codeword whose data shards are
        every rank's staging slot `slot` (K ++ V, half bytes each)."""
        self._barrier(device)  # every rank's staging write precedes every peer read
        plan = self._plan(slot, half, device)
        spec, lo, hi = plan["spec"], plan["lo"], plan["hi"]
        # parity buffers alternate with the staging slot; before overwriting one,
        # wait only for the host copy that last read it (not for the copy stream)
        if self._parity_free[slot] is not None:
            torch.cuda.current_stream(device).wait_event(self._parity_free[slot])
        e0, e1 = self._event(), self._event()
        e0.record()
        if plan["enc"] is not None:
            plan["enc"]()
        e1.record()
        rec = self._record(chunk_id, -1, None, None, None, spec.m * (hi - lo))
        rec["slice"] = [lo, hi]
        rec["scheme"] = spec.scheme
        if self.cfg.offload and hi > lo:
            entry = dict(lo=lo, hi=hi, half=half, spec=spec)
            self._parity_free[slot] = self._offload(rec, plan["views"], e0, e1, entry)
        else:
            self._pending.append((rec, None, e0, e1))
        self._drain(block=False)
        return plan["views"], (lo, hi)

    def _copies_landed(self):
        """The store's block is written by raw copies the allocator does not
        track: let them land before the block can be released."""
        if self._copy_stream is not None:
            self._copy_stream.synchronize()

    def _offload(self, rec, parity, e0, e1, entry):
        """Copy this rank's parity slice to its pinned host slot on a side stream;
        returns the event after which the device parity buffer may be overwritten."""
        dev = parity[0].device
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(dev)
        nbytes = sum(t.numel() for t in parity)
        stored = self._store.put(rec["chunk_id"], nbytes)
        host = stored["host"]
        cs = self._copy_stream
        ready = self._event()
        ready.record(torch.cuda.current_stream(dev))
        cs.wait_event(ready)
        self._events.append(ready)  # a later record does not change the wait already enqueued
        d0 = self._event()
        d1 = torch.cuda.Event(enable_timing=True)  # kept by the store entry: not pooled
        d0.record(cs)
        dst, copy = host.data_ptr(), _lib.lib().gsec_copy_async
        for t in parity:  # raw stream-ordered copies: no per-copy framework bookkeeping
            _lib.check(copy(dst, t.data_ptr(), t.numel(), cs.cuda_stream))
            dst += t.numel()
        d1.record(cs)
        stored.update(entry, copied=d1)
        self._pending.append((rec, (d0, d1), e0, e1))
        return d1

    def _drain(self, block: bool):
        keep = []
        for rec, d2h, e0, e1 in self._pending:
            if not block and not e1.query():
                keep.append((rec, d2h, e0, e1))
                continue
            if block:
                e1.synchronize()
            rec["timings"]["rdp_encode_ms"] = float(e0.elapsed_time(e1))
            if d2h is not None:
                if not block and not d2h[1].query():
                    keep.append((rec, d2h, e0, e1))
                    continue
                d2h[1].synchronize()
                rec["timings"]["gpu_to_cpu_ms"] = float(d2h[0].elapsed_time(d2h[1]))
                self._events.append(d2h[0])
            self._events += [e0, e1]
            self._emit(rec)
        self._pending = keep

    def flush(self):
        """Wait for outstanding encodes/offloads and emit their records."""
        self._drain(block=True)

    def close(self):
        self.flush()
        if self._peers is not None:
            dev = self._staging[0][0].device
            self._barrier(dev)
            torch.cuda.synchronize(dev)
            self._peers.close()
            self._peers = None

    # ------------------------------------------------------------ metrics ----
    def _record(self, chunk_id, dst_rank, enc_ms, d2h_ms, h2d_ms, parity_bytes):
        return {
            "chunk_id": int(chunk_id),
            "dst_rank": int(dst_rank),
            "first_chunk_wall_ms": None if self.first_chunk_wall_ms is None else float(self.first_chunk_wall_ms),
            "timings": {"rdp_encode_ms": enc_ms, "rdp_decode_ms": None, "gpu_to_cpu_ms": d2h_ms,
                        "cpu_to_gpu_ms": h2d_ms, "parity_bytes": int(parity_bytes)},
        }

    def _emit(self, rec):
        self.records.append(rec)
        if self.cfg.metrics_file:
            try:
                with open(self.cfg.metrics_file, "a", encoding="utf-8") as f:
                    f.write(json.dumps(rec) + "\n")
            except Exception:
                pass
        if self.cfg.verbose:
            t = rec["timings"]
            _log(f"chunk={rec['chunk_id']} dst={rec['dst_rank']} encode={t['rdp_encode_ms']}ms "
                 f"D2H={t['gpu_to_cpu_ms']}ms parity={t['parity_bytes'] / 2**20:.3f}MiB")

    # ------------------------------------------------------------ the hook --
    def on_extend(self, batch, kv_pool) -> None:
        """Protect the delta KV of one extend call (bench_ghostserve_rdp.py:428-471)."""
        if not (dist.is_available() and dist.is_initialized()):
            return
        slots = getattr(batch, "slot_mapping", None)
        if slots is None:
            return
        if not isinstance(slots, torch.Tensor):
            slots = torch.as_tensor(slots, device=kv_pool.device)
        if self.cfg.mode != "reference":
            # the pool is read through the slot list on the device: no host sync
            if slots.numel() == 0:
                return
            if self.cfg.protect == "chunk":
                # one codeword per prefill chunk: remember this layer's pool and
                # encode after the chunk's last layer call
                if self.cfg.chunk_layers < 1:
                    raise ValueError("protect='chunk' needs chunk_layers (the model's layer count)")
                self._chunk_pools.append(kv_pool)
                if len(self._chunk_pools) < self.cfg.chunk_layers:
                    return
                pools, self._chunk_pools = self._chunk_pools, []
            else:
                pools = [kv_pool]
            chunk_id, _ = self.next_chunk_id(device=kv_pool.device)
            if self.first_chunk_wall_ms is None and self.cfg.prog_start_mono == self.cfg.prog_start_mono:
                self.first_chunk_wall_ms = (time.perf_counter() - self.cfg.prog_start_mono) * 1000.0
            self.encode_pools(pools, slots.contiguous(), chunk_id)
            return
        active = slots != -1
        if int(active.sum().item()) == 0:
            return
        active_slots = slots[active].to(dtype=torch.long)
        local_k = kv_pool[active_slots, 0].contiguous()
        local_v = kv_pool[active_slots, 1].contiguous()
        chunk_id, dst_rank = self.next_chunk_id(device=local_k.device)
        if self.first_chunk_wall_ms is None and self.cfg.prog_start_mono == self.cfg.prog_start_mono:
            self.first_chunk_wall_ms = (time.perf_counter() - self.cfg.prog_start_mono) * 1000.0
        gathered = self.gather_kv(local_k, local_v, dst_rank)
        if gathered is not None:
            self.compute_parity_to_cpu(*gathered, chunk_id, dst_rank)


def patch_backend(backend, ft: KVFaultTolerance) -> bool:
    """_patch_flashinfer_backend, bench_ghostserve_rdp.py:396-481."""
    if getattr(backend, "_gsec_patched", False):
        return True
    if "FlashInfer" not in backend.__class__.__name__:
        _log(f"SKIP: backend is {backend.__class__.__name__}, not FlashInfer")
        return False
    if not hasattr(backend, "forward_extend"):
        _log("SKIP: FlashInfer backend missing forward_extend")
        return False
    orig = backend.forward_extend

    @functools.wraps(orig)
    def hooked_forward_extend(*args, **kwargs):
        res = orig(*args, **kwargs)
        try:
            batch = kwargs.get("batch", None)
            if batch is None and len(args) >= 1:
                batch = args[0]
            if batch is None:
                return res
            # The reference chains these with `or` (bench_ghostserve_rdp.py:441), which
            # asks a multi-element tensor for its truth value and raises, so its hook
            # gives up whenever the pool is found as kv_buffer or kv_pool.
            kv_pool = None
            for name in ("kv_buffer", "kv_pool", "kv_cache"):
                kv_pool = getattr(backend, name, None)
                if kv_pool is not None:
                    break
            if kv_pool is None:
                return res
            ft.on_extend(batch, kv_pool)
        except Exception as e:  # the hook never breaks the model's forward pass
            _log(f"FlashInfer hook error: {e}")
        return res

    backend.forward_extend = hooked_forward_extend
    backend._gsec_patched = True
    _log("Successfully hooked FlashInferAttnBackend.forward_extend")
    return True


def patch_model_runner(model_runner, ft: KVFaultTolerance) -> bool:
    """Find the attention backend of a ModelRunner and patch it (:405-411)."""
    backend = getattr(model_runner, "attn_backend", None) or getattr(model_runner, "attention_backend", None)
    if backend is None:
        return False
    return patch_backend(backend, ft)
