"""Host-resident shards: pipelined host -> device -> encode/decode -> host.

The reference hook copies P and Q to the host after every chunk with blocking
copies (bench_ghostserve_rdp.py:362-374) and has no restore path
(``rdp_decode_ms`` is always None, :383).  ``HostPipeline`` streams shards that
live in pinned host memory through a small ring of device staging slots:

    stream h2d : copy chunk c of every input shard into slot c % S
    stream comp: encode (or decode) slot c on the GPU
    stream d2h : copy chunk c of every output shard back to the host

so PCIe transfers in both directions overlap the kernels of neighbouring
chunks.  One ``cudaMemcpyAsync`` per shard per chunk; no device sync inside.
Chunks are whole RDP stripes (or multiples of 16 bytes for XOR/RS8).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from . import codec


class HostPipeline:
    def __init__(self, spec: codec.CodeSpec, data_bytes: int, chunk_bytes: int = 4 << 20, slots: int = 3,
                 device: Optional[torch.device] = None):
        if data_bytes % 16:
            raise ValueError("data_bytes must be a multiple of 16")
        self.spec = spec
        self.data_bytes = data_bytes
        self.parity_bytes = spec.parity_bytes(data_bytes)
        g = spec.stripe_bytes()
        self.chunk = max(g, chunk_bytes // g * g)
        self.nchunks = -(-self.parity_bytes // self.chunk)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.slots = max(2, slots)
        n = spec.n
        self.buf = [[torch.empty(self.chunk, dtype=torch.uint8, device=self.device) for _ in range(n)]
                    for _ in range(self.slots)]
        self.s_h2d = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_d2h = torch.cuda.Stream(self.device)
        self.ev_in = [torch.cuda.Event() for _ in range(self.slots)]
        self.ev_done = [torch.cuda.Event() for _ in range(self.slots)]
        self.ev_free = [torch.cuda.Event() for _ in range(self.slots)]
        self.launches = 0
        self._next = 0          # staging slots are used round-robin across calls
        self._used = [False] * self.slots
        self._joined = True     # the last call ended by joining the current stream

    def _range(self, c: int):
        lo = c * self.chunk
        return lo, min(lo + self.chunk, self.parity_bytes), min(lo + self.chunk, self.data_bytes)

    def _run(self, inputs, outputs, work, join: bool):
        """inputs/outputs: lists of (shard index, host tensor); work(slot, nbytes_data, pbytes).

        After a call with join=False the next call is not ordered after it on
        the current stream: its copies in start as soon as staging slots free
        up, overlapping the previous call's last kernels and copies out."""
        cur = torch.cuda.current_stream(self.device)
        if self._joined:
            for s in (self.s_h2d, self.s_comp, self.s_d2h):
                s.wait_stream(cur)
        for c in range(self.nchunks):
            sl = self._next % self.slots
            self._next += 1
            lo, hi_p, hi_d = self._range(c)
            with torch.cuda.stream(self.s_h2d):
                if self._used[sl]:
                    self.s_h2d.wait_event(self.ev_free[sl])
                self._used[sl] = True
                for idx, h in inputs:
                    hi = hi_d if idx < self.spec.k else hi_p
                    if hi > lo:
                        self.buf[sl][idx][:hi - lo].copy_(h[lo:hi], non_blocking=True)
                self.ev_in[sl].record(self.s_h2d)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(self.ev_in[sl])
                work(sl, max(hi_d - lo, 0), hi_p - lo)
                self.ev_done[sl].record(self.s_comp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(self.ev_done[sl])
                for idx, h in outputs:
                    hi = hi_d if idx < self.spec.k else hi_p
                    if hi > lo:
                        h[lo:hi].copy_(self.buf[sl][idx][:hi - lo], non_blocking=True)
                self.ev_free[sl].record(self.s_d2h)
        self._joined = join
        if join:
            cur.wait_stream(self.s_d2h)

    def join(self) -> None:
        """Order the current stream after every call made so far."""
        torch.cuda.current_stream(self.device).wait_stream(self.s_d2h)
        self._joined = True

    def encode(self, host_data: Sequence[torch.Tensor], host_parity: Sequence[torch.Tensor],
               join: bool = True) -> None:
        """Enqueue the encode of pinned host shards. Parity lands in host_parity;
        with join (the default) it is ordered before later work on the current
        stream, otherwise after the next join() (or joining call). Host inputs
        must be ready when the call is made."""
        k = self.spec.k

        def work(sl, nd, np_):
            # every chunk holds data: parity pads less than one stripe past data_bytes
            data = [self.buf[sl][i][:nd] for i in range(k)]
            par = [self.buf[sl][k + j] for j in range(self.spec.m)]
            codec.encode_ptrs(self.spec, [t.data_ptr() for t in data], None, nd, nd,
                              [t.data_ptr() for t in par], 0, np_, int(self.s_comp.cuda_stream))
            self.launches += 1

        self._run([(i, host_data[i]) for i in range(k)],
                  [(k + j, host_parity[j]) for j in range(self.spec.m)], work, join)

    def decode(self, host_shards: List[torch.Tensor], erased: Sequence[int], join: bool = True) -> None:
        """Enqueue the rebuild of ``erased`` host shards (in place) from the
        surviving host shards (join as for encode)."""
        erased = list(erased)
        k = self.spec.k
        alive = [i for i in range(self.spec.n) if i not in erased]

        def work(sl, nd, np_):
            ptrs = [self.buf[sl][i].data_ptr() for i in range(self.spec.n)]
            codec.decode_ptrs(self.spec, ptrs, None, nd, nd, erased, 0, np_, int(self.s_comp.cuda_stream))
            self.launches += 1

        self._run([(i, host_shards[i]) for i in alive], [(e, host_shards[e]) for e in erased], work, join)
