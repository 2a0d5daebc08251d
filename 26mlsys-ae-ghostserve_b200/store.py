"""Host store of parity slices, keyed by chunk id (host-side logic only).

The hook keeps every chunk's parity slice in host memory so that a lost rank's
KV can be rebuilt later; the reference copies P and Q to the host and drops
them (bench_ghostserve_rdp.py:362-372). Slices live in a byte ring over one
block (pinned, for asynchronous device copies, when ``pin``): chunks of any
size take consecutive byte ranges, wrapping at the end, and the chunks whose
bytes a new one overwrites are dropped (they are the oldest in the block). At
most ``keep`` chunks are kept. A block is only replaced by a larger one when a
chunk does not fit; chunks in the replaced block stay readable until they are
dropped by count. A chunk id stored again with the same size reuses its bytes.
"""
from __future__ import annotations

from collections import OrderedDict, deque
from typing import Callable, Optional

import torch


class ParityStore:
    def __init__(self, keep: int, budget: int, pin: bool = True,
                 before_release: Optional[Callable[[], None]] = None):
        self.keep = max(1, int(keep))
        self.budget = int(budget)
        self.pin = pin
        self.before_release = before_release  # called before the block may be freed
        self._entries: "OrderedDict[int, dict]" = OrderedDict()  # oldest first
        self._block = None
        self._gen = 0
        self._head = 0
        self._ring = deque()  # this block's entries in ring (= address) order

    # ---------------------------------------------------------------- queries
    def get(self, cid: int):
        return self._entries.get(cid)

    def __getitem__(self, cid: int) -> dict:
        return self._entries[cid]

    def __contains__(self, cid: int) -> bool:
        return cid in self._entries

    def __len__(self) -> int:
        return len(self._entries)

    def keys(self):
        return list(self._entries)

    @property
    def block_bytes(self) -> int:
        return 0 if self._block is None else self._block.numel()

    # ---------------------------------------------------------------- updates
    def put(self, cid: int, nbytes: int) -> dict:
        """Reserve nbytes for chunk cid; returns its entry (``host`` = the byte
        view to fill; the caller may add fields)."""
        old = self._entries.pop(cid, None)
        if old is not None and old["gen"] == self._gen and old["size"] == nbytes:
            entry = dict(cid=cid, gen=old["gen"], off=old["off"], size=nbytes, host=old["host"])
            self._ring = deque(entry if e is old else e for e in self._ring)
        else:
            host, off = self._alloc(nbytes)
            entry = dict(cid=cid, gen=self._gen, off=off, size=nbytes, host=host)
            self._ring.append(entry)
        while len(self._entries) >= self.keep:
            self._entries.popitem(last=False)
        self._entries[cid] = entry
        return entry

    def _alloc(self, nbytes: int):
        if self._block is None or nbytes > self._block.numel():
            if self._block is not None and self.before_release is not None:
                self.before_release()
            size = max(4 * nbytes, min(self.budget, self.keep * nbytes), 16)
            self._block = torch.empty(size, dtype=torch.uint8, pin_memory=self.pin)
            self._gen += 1
            self._head = 0
            self._ring.clear()
        if self._head + nbytes > self._block.numel():
            # wrap: the chunks between the head and the block's end are the oldest
            # (an earlier lap's); drop them so the ring stays in address order
            while self._ring and self._ring[0]["off"] >= self._head:
                self._drop(self._ring.popleft())
            self._head = 0
        lo, hi = self._head, self._head + nbytes
        # the entries these bytes overwrite are at the front of the ring
        while self._ring and self._ring[0]["off"] < hi and lo < self._ring[0]["off"] + self._ring[0]["size"]:
            self._drop(self._ring.popleft())
        self._head = hi
        return self._block[lo:hi], lo

    def _drop(self, gone: dict) -> None:
        if self._entries.get(gone["cid"]) is gone:  # not already dropped by count or replaced
            del self._entries[gone["cid"]]
