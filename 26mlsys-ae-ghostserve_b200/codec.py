"""Engine API: encode / decode erasure-code shards that live in GPU memory.

A *shard* is one rank's KV bytes (any dtype, read as raw bytes).  Data shards
may be given as one tensor or as a ``(lo, hi)`` pair of tensors — e.g. a rank's
K and V buffers — which the kernels read as ``lo ++ hi`` without a copy.

Codes (``CodeSpec``):

* ``xor``  k data + 1 parity, byte-wise XOR;
* ``rdp``  Row-Diagonal Parity, p prime, k <= p-1 data + row parity P +
  diagonal parity Q, stripes of (p-1) units of ``unit`` bytes (4 KiB default);
* ``rs8``  Reed-Solomon over GF(2^8)/0x11d with a Cauchy generator, k data + m.

All calls are stream-ordered on the current torch stream (or ``stream``) and
do not synchronise.  The work is done by libgsec (hand-written sm_100a
kernels); there is no CPU path.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple, Union

import torch

from . import _lib

SUPPORTED_PRIMES = (3, 5, 7, 11, 13, 17)

ShardLike = Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]


@dataclass(frozen=True)
class CodeSpec:
    scheme: str
    k: int
    m: int
    p: int = 0
    unit: int = 4096

    @staticmethod
    def xor(k: int) -> "CodeSpec":
        return CodeSpec("xor", k, 1)

    @staticmethod
    def rdp(k: int, p: Optional[int] = None, unit: int = 4096) -> "CodeSpec":
        if p is None:
            p = next((q for q in SUPPORTED_PRIMES if q - 1 >= k), None)
            if p is None:
                raise ValueError(f"RDP supports at most {SUPPORTED_PRIMES[-1] - 1} data shards")
        return CodeSpec("rdp", k, 2, p, unit)

    @staticmethod
    def rs8(k: int, m: int = 2) -> "CodeSpec":
        return CodeSpec("rs8", k, m)

    @property
    def n(self) -> int:
        return self.k + self.m

    def c_code(self) -> _lib.Code:
        scheme = {"xor": _lib.SCHEME_XOR, "rdp": _lib.SCHEME_RDP, "rs8": _lib.SCHEME_RS8}[self.scheme]
        return _lib.Code(scheme, self.k, self.m, self.p, self.unit)

    def stripe_bytes(self) -> int:
        return (self.p - 1) * self.unit if self.scheme == "rdp" else 16

    def parity_bytes(self, data_bytes: int) -> int:
        if self.scheme == "rdp":
            sb = self.stripe_bytes()
            return -(-data_bytes // sb) * sb
        return data_bytes


def stream_handle(stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def _check_tensor(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")


def _split_shards(shards: Sequence[ShardLike], what: str):
    """-> (lo_ptrs, hi_ptrs or None, split, nbytes)."""
    los, his, split, total = [], [], None, None
    for i, s in enumerate(shards):
        if isinstance(s, (tuple, list)):
            lo, hi = s
            _check_tensor(lo, f"{what}[{i}].lo")
            _check_tensor(hi, f"{what}[{i}].hi")
            sp, tot = _nbytes(lo), _nbytes(lo) + _nbytes(hi)
            los.append(lo.data_ptr())
            his.append(hi.data_ptr())
        else:
            _check_tensor(s, f"{what}[{i}]")
            sp, tot = None, _nbytes(s)
            los.append(s.data_ptr())
            his.append(None)
        if total is None:
            total, split = tot, sp
        elif tot != total or sp != split:
            raise ValueError(f"{what}: all shards must have the same size and split")
    two_seg = split is not None
    if not two_seg:
        his = None
    return los, his, (split if two_seg else total), total


def encode_ptrs(spec: CodeSpec, data_lo: Sequence[int], data_hi: Optional[Sequence[int]], split: int,
                data_bytes: int, parity: Sequence[int], begin: int = 0, end: Optional[int] = None,
                stream: Optional[int] = None) -> None:
    """Raw-pointer encode (pointers may be peer-mapped); see gsec_encode."""
    if end is None:
        end = spec.parity_bytes(data_bytes)
    code = spec.c_code()
    _lib.call("gsec_encode", _lib.C.byref(code), _lib.ptr_array(data_lo),
              _lib.ptr_array(data_hi) if data_hi is not None else None, int(split), int(data_bytes),
              _lib.ptr_array(parity), int(begin), int(end),
              _lib.C.c_void_p(stream if stream is not None else stream_handle()))


def decode_ptrs(spec: CodeSpec, shard_lo: Sequence[int], shard_hi: Optional[Sequence[int]], split: int,
                data_bytes: int, erased: Sequence[int], begin: int = 0, end: Optional[int] = None,
                stream: Optional[int] = None) -> None:
    """Raw-pointer decode (pointers may be peer-mapped); see gsec_decode."""
    if end is None:
        end = spec.parity_bytes(data_bytes)
    code = spec.c_code()
    _lib.call("gsec_decode", _lib.C.byref(code), _lib.ptr_array(shard_lo),
              _lib.ptr_array(shard_hi) if shard_hi is not None else None, int(split), int(data_bytes),
              _lib.i32_array(erased), len(erased), int(begin), int(end),
              _lib.C.c_void_p(stream if stream is not None else stream_handle()))


def _pool_geometry(pool: torch.Tensor, plane: int):
    """(row bytes, slot pitch, plane byte offset) of a KV pool [slots, planes, ...]."""
    if not isinstance(pool, torch.Tensor) or not pool.is_cuda or pool.dim() < 2:
        raise ValueError("pool must be a CUDA tensor [slots, planes, ...]")
    if not 0 <= plane < pool.shape[1]:
        raise ValueError(f"plane {plane} out of range for a pool of {pool.shape[1]} planes")
    if not pool[0, 0].is_contiguous():
        raise ValueError("a pool row (pool[slot, plane]) must be contiguous")
    es = pool.element_size()
    return pool[0, 0].numel() * es, pool.stride(0) * es, plane * pool.stride(1) * es


def _slot_list(slots: torch.Tensor, device) -> torch.Tensor:
    if not isinstance(slots, torch.Tensor) or slots.device != device:
        raise ValueError("slots must be a tensor on the pool's device")
    if slots.dtype not in (torch.int32, torch.int64) or not slots.is_contiguous():
        raise ValueError("slots must be a contiguous int32 or int64 tensor")
    return slots


def slots_gather(pool: torch.Tensor, slots: torch.Tensor, out: torch.Tensor, plane: int = 0,
                 stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out[i] = pool[slots[i], plane] for every list position (zero rows for
    negative slots), as bytes: out holds len(slots) rows back to back."""
    row, pitch, off = _pool_geometry(pool, plane)
    slots = _slot_list(slots, pool.device)
    n = slots.numel()
    _check_tensor(out, "out")
    if _nbytes(out) < n * row:
        raise ValueError(f"out holds {_nbytes(out)} bytes, needs {n * row}")
    _lib.call("gsec_slots_gather", pool.data_ptr() + off, pitch, 0, 1, row, slots.data_ptr(),
              slots.element_size(), n, pool.shape[0], out.data_ptr(), stream_handle(stream))
    return out


def slots_scatter(pool: torch.Tensor, slots: torch.Tensor, src: torch.Tensor, plane: int = 0,
                  stream: Optional[torch.cuda.Stream] = None) -> None:
    """Inverse of slots_gather: pool[slots[i], plane] = src row i (negative slots skipped)."""
    row, pitch, off = _pool_geometry(pool, plane)
    slots = _slot_list(slots, pool.device)
    n = slots.numel()
    _check_tensor(src, "src")
    if _nbytes(src) < n * row:
        raise ValueError(f"src holds {_nbytes(src)} bytes, needs {n * row}")
    _lib.call("gsec_slots_scatter", pool.data_ptr() + off, pitch, 0, 1, row, slots.data_ptr(),
              slots.element_size(), n, pool.shape[0], src.data_ptr(), stream_handle(stream))


class PreparedEncode:
    """One gsec_encode call with its arguments marshalled once.

    For loops that encode the same buffers repeatedly (every prefill chunk of
    the hook, the benchmark): calling it costs one ctypes call (~3 us of host
    time) instead of rebuilding the pointer arrays each time."""

    def __init__(self, spec: CodeSpec, data_lo: Sequence[int], data_hi: Optional[Sequence[int]], split: int,
                 data_bytes: int, parity: Sequence[int], begin: int = 0, end: Optional[int] = None,
                 stream: Optional[int] = None):
        self._fn = _lib.lib().gsec_encode
        self._code = spec.c_code()
        self._args = (_lib.C.byref(self._code), _lib.ptr_array(data_lo),
                      _lib.ptr_array(data_hi) if data_hi is not None else None, int(split), int(data_bytes),
                      _lib.ptr_array(parity), int(begin), int(spec.parity_bytes(data_bytes) if end is None else end),
                      _lib.C.c_void_p(stream if stream is not None else stream_handle()))

    def __call__(self) -> None:
        _lib.check(self._fn(*self._args))


class PreparedDecode:
    """One gsec_decode call with its arguments marshalled once."""

    def __init__(self, spec: CodeSpec, shard_lo: Sequence[int], shard_hi: Optional[Sequence[int]], split: int,
                 data_bytes: int, erased: Sequence[int], begin: int = 0, end: Optional[int] = None,
                 stream: Optional[int] = None):
        self._fn = _lib.lib().gsec_decode
        self._code = spec.c_code()
        self._args = (_lib.C.byref(self._code), _lib.ptr_array(shard_lo),
                      _lib.ptr_array(shard_hi) if shard_hi is not None else None, int(split), int(data_bytes),
                      _lib.i32_array(erased), len(erased), int(begin),
                      int(spec.parity_bytes(data_bytes) if end is None else end),
                      _lib.C.c_void_p(stream if stream is not None else stream_handle()))

    def __call__(self) -> None:
        _lib.check(self._fn(*self._args))


def encode(spec: CodeSpec, data: Sequence[ShardLike], parity: Optional[List[torch.Tensor]] = None,
           begin: int = 0, end: Optional[int] = None,
           stream: Optional[torch.cuda.Stream] = None) -> List[torch.Tensor]:
    """Compute the m parity shards of ``data`` (k shards). Returns the parity
    tensors (uint8, ``spec.parity_bytes(data_bytes)`` each)."""
    if len(data) != spec.k:
        raise ValueError(f"expected {spec.k} data shards, got {len(data)}")
    los, his, split, nbytes = _split_shards(data, "data")
    pbytes = spec.parity_bytes(nbytes)
    dev = (data[0][0] if isinstance(data[0], (tuple, list)) else data[0]).device
    if parity is None:
        parity = [torch.empty(pbytes, dtype=torch.uint8, device=dev) for _ in range(spec.m)]
    if len(parity) != spec.m:
        raise ValueError(f"expected {spec.m} parity buffers")
    for j, t in enumerate(parity):
        _check_tensor(t, f"parity[{j}]")
        if _nbytes(t) < pbytes:
            raise ValueError(f"parity[{j}] holds {_nbytes(t)} bytes, needs {pbytes}")
    encode_ptrs(spec, los, his, split, nbytes, [t.data_ptr() for t in parity], begin, end,
                stream_handle(stream))
    return parity


def decode(spec: CodeSpec, shards: List[Optional[ShardLike]], erased: Sequence[int],
           data_bytes: Optional[int] = None, begin: int = 0, end: Optional[int] = None,
           stream: Optional[torch.cuda.Stream] = None) -> List[ShardLike]:
    """Rebuild the ``erased`` shards of a k+m list (data..., parity...).

    Surviving entries are read; erased entries are written in place, or
    allocated when they are ``None``.  Returns the completed list."""
    if len(shards) != spec.n:
        raise ValueError(f"expected {spec.n} shards, got {len(shards)}")
    erased = [int(e) for e in erased]
    ref = next((s for i, s in enumerate(shards) if i < spec.k and s is not None), None)
    if data_bytes is None:
        if ref is None:
            raise ValueError("data_bytes is required when every data shard is missing")
        data_bytes = sum(_nbytes(t) for t in ref) if isinstance(ref, (tuple, list)) else _nbytes(ref)
    pbytes = spec.parity_bytes(data_bytes)
    any_t = next(t for t in shards if t is not None)
    dev = (any_t[0] if isinstance(any_t, (tuple, list)) else any_t).device
    out = list(shards)
    for e in erased:
        if out[e] is None:
            out[e] = torch.empty(data_bytes if e < spec.k else pbytes, dtype=torch.uint8, device=dev)
    data = out[:spec.k]
    los, his, split, nbytes = _split_shards(data, "data")
    if nbytes != data_bytes:
        raise ValueError("data shard size does not match data_bytes")
    for j in range(spec.m):
        t = out[spec.k + j]
        _check_tensor(t, f"parity[{j}]")
        if _nbytes(t) < pbytes:
            raise ValueError(f"parity[{j}] holds {_nbytes(t)} bytes, needs {pbytes}")
        los.append(t.data_ptr())
        if his is not None:
            his.append(None)
    decode_ptrs(spec, los, his, split, data_bytes, erased, begin, end, stream_handle(stream))
    return out


def device_status(clear: bool = True) -> int:
    """Synchronise the current device and return its libgsec status word
    (0 = every bounded wait since the last clear completed)."""
    v = _lib.C.c_uint32(0)
    _lib.call("gsec_device_status", _lib.C.byref(v), int(bool(clear)))
    return int(v.value)


def parity_bytes(spec: CodeSpec, data_bytes: int) -> int:
    """Parity shard size as computed by the library (no GPU needed)."""
    out = _lib.C.c_int64(0)
    code = spec.c_code()
    _lib.call("gsec_parity_bytes", _lib.C.byref(code), int(data_bytes), _lib.C.byref(out))
    return int(out.value)
