"""Extension-level names of the reference, backed by libgsec.

The reference JIT-builds four torch extensions and calls them from Python.  The
objects here expose the same function names and argument order, so code that
called the reference extension calls these instead:

* ``xor_kernel``  <- benchmark/xor/kernel.cu:225-244
* ``rdp_kernel``  <- benchmark/rdp/kernel.cu:525-538
* ``rs_kernel``   <- benchmark/rs/kernel.cu:314-320
* ``rdp_kv_ops``  <- bench_ghostserve_rdp.py:201-206 (the hook's extension)

Differences, all documented at each function: the GF tables arguments of the
RS functions are accepted and ignored (the library derives the same tables),
index tensors are read on the host, and every launch is on the current torch
stream instead of the legacy default stream.
"""
from __future__ import annotations

import torch

from . import _lib
from .codec import stream_handle


def _ptr(t: torch.Tensor):
    return _lib.C.c_void_p(t.data_ptr())


def _s():
    return _lib.C.c_void_p(stream_handle())


def _rows(t: torch.Tensor, what: str):
    """(pointer, pitch in elements) of a 2-D row-major tensor with unit inner stride."""
    if not t.is_cuda:
        raise ValueError(f"{what} must be a CUDA tensor")
    if t.dim() == 1:
        return t.data_ptr(), t.numel()
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{what} must be [rows, cols] with unit column stride")
    return t.data_ptr(), t.stride(0)


def _check_cuda(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("All tensors must be on CUDA")


class _XorKernel:
    """xor_kernel (benchmark/xor/kernel.cu)."""

    @staticmethod
    def encode_xor(data_padded: torch.Tensor, shards: torch.Tensor, data_shards: int, shard_size: int) -> None:
        """encode_xor_launcher, benchmark/xor/kernel.cu:158-171."""
        _check_cuda(data_padded, shards)
        p, pitch = _rows(shards, "shards")
        if shards.dim() == 1:
            pitch = int(shard_size)
        _lib.call("gsec_xor_encode", _ptr(data_padded), _lib.C.c_void_p(p), int(data_shards), int(shard_size),
                  int(pitch), _s())

    @staticmethod
    def reconstruct_xor(encoded_data: torch.Tensor, recovered_data: torch.Tensor,
                        recovered_missing_shards: torch.Tensor, shard_size: int, data_shards: int,
                        missing_indices: torch.Tensor) -> None:
        """reconstruct_xor_launcher, benchmark/xor/kernel.cu:173-191. The reference
        reads encoded_data and writes recovered_data (its caller passes the same
        tensor, benchmark/xor/main.py:174-177); here encoded_data must equal
        recovered_data or hold the same bytes."""
        _check_cuda(encoded_data, recovered_data, recovered_missing_shards)
        if recovered_data.data_ptr() != encoded_data.data_ptr():
            recovered_data.copy_(encoded_data)
        p, pitch = _rows(recovered_data, "recovered_data")
        if recovered_data.dim() == 1:
            pitch = int(shard_size)
        missing = [int(x) for x in missing_indices.reshape(-1).tolist()]
        _lib.call("gsec_xor_reconstruct", _lib.C.c_void_p(p), _ptr(recovered_missing_shards), int(shard_size),
                  int(pitch), int(data_shards), _lib.i32_array(missing), len(missing), _s())

    @staticmethod
    def pack_kv(key_input: torch.Tensor, value_input: torch.Tensor, kv_bytes: torch.Tensor, n: int,
                seq_len: int) -> None:
        """pack_kv_launcher, benchmark/xor/kernel.cu:193-207."""
        _check_cuda(key_input, value_input, kv_bytes)
        half = 2 * int(seq_len) * int(n)
        _lib.call("gsec_rows_pack", _ptr(key_input), half, _ptr(value_input), half, _ptr(kv_bytes), 2 * half,
                  2 * half, 1, _s())

    @staticmethod
    def unpack_kv(kv_bytes: torch.Tensor, dequant_KV: torch.Tensor, n: int, seq_len: int) -> None:
        """unpack_kv_launcher, benchmark/xor/kernel.cu:209-223 (which also
        synchronises the device; so does this)."""
        _check_cuda(kv_bytes, dequant_KV)
        total = 4 * int(seq_len) * int(n)
        _lib.call("gsec_rows_unpack", _ptr(kv_bytes), total, total, 1, _ptr(dequant_KV), total, None, 0, _s())
        torch.cuda.synchronize()


class _RdpKernel:
    """rdp_kernel_rdp_parallel (benchmark/rdp/kernel.cu)."""

    @staticmethod
    def fused_backup_full_kv(K_TN, V_TN, shards, num_data_shards, shard_size, T, n, star_base) -> None:
        """fused_backup_full_kv_launcher, benchmark/rdp/kernel.cu:366-395."""
        _check_cuda(K_TN, V_TN, shards)
        p, pitch = _rows(shards, "shards")
        _lib.call("gsec_rdpref_backup", _ptr(K_TN), _ptr(V_TN), _lib.C.c_void_p(p), int(pitch),
                  int(num_data_shards), int(shard_size), int(T), int(n), int(star_base), _s())

    @staticmethod
    def fused_recovery_full_kv(shards, out_half_TN, num_data_shards, shard_size, T, n, star_base, missing_a,
                               missing_b) -> None:
        """fused_recovery_full_kv_launcher, benchmark/rdp/kernel.cu:397-521."""
        _check_cuda(shards, out_half_TN)
        p, pitch = _rows(shards, "shards")
        _lib.call("gsec_rdpref_recovery", _lib.C.c_void_p(p), int(pitch), _ptr(out_half_TN),
                  int(num_data_shards), int(shard_size), int(T), int(n), int(star_base), int(missing_a),
                  int(missing_b), _s())


class _RsKernel:
    """rs_kernel16 (benchmark/rs/kernel.cu)."""

    @staticmethod
    def pack_fp16_pair_to_u16(k: torch.Tensor, v: torch.Tensor, out: torch.Tensor) -> None:
        """benchmark/rs/kernel.cu:225-243."""
        _check_cuda(k, v, out)
        nk, nv = 2 * k.numel(), 2 * v.numel()
        _lib.call("gsec_rows_pack", _ptr(k), nk, _ptr(v), nv, _ptr(out), nk + nv, nk + nv, 1, _s())

    @staticmethod
    def u16_to_fp16_split(inp: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor, N_k: int, N_v: int) -> None:
        """benchmark/rs/kernel.cu:245-263."""
        _check_cuda(inp, k_out, v_out)
        nk, nv = 2 * int(N_k), 2 * int(N_v)
        _lib.call("gsec_rows_unpack", _ptr(inp), nk + nv, nk + nv, 1, _ptr(k_out), nk, _ptr(v_out), nv, _s())

    @staticmethod
    def encode_rs_u16(data_padded, shards, data_shards, parity_shards, shard_size, gf_exp=None, gf_log=None) -> None:
        """encode_rs_u16, benchmark/rs/kernel.cu:265-285 (tables ignored)."""
        _check_cuda(data_padded, shards)
        p, pitch = _rows(shards, "shards")
        _lib.call("gsec_rs16_encode", _ptr(data_padded), _lib.C.c_void_p(p), int(pitch), int(data_shards),
                  int(parity_shards), int(shard_size), _s())

    @staticmethod
    def reconstruct_rs_u16_inplace(shards, shard_size, data_shards, parity_shards, missing_data, parity_used,
                                   gf_exp=None, gf_log=None) -> None:
        """reconstruct_rs_u16_inplace, benchmark/rs/kernel.cu:287-312 (tables
        ignored; index tensors read on the host)."""
        _check_cuda(shards)
        p, pitch = _rows(shards, "shards")
        md = [int(x) for x in missing_data.reshape(-1).tolist()]
        pu = [int(x) for x in parity_used.reshape(-1).tolist()]
        _lib.call("gsec_rs16_reconstruct", _lib.C.c_void_p(p), int(pitch), int(shard_size), int(data_shards),
                  int(parity_shards), _lib.i32_array(md), len(md), _lib.i32_array(pu), _s())


class _RdpKvOps:
    """rdp_kv_ops, the hook's extension (bench_ghostserve_rdp.py:92-207)."""

    @staticmethod
    def pack_row_from_block(k_blk: torch.Tensor, v_blk: torch.Tensor, shards: torch.Tensor, row: int) -> None:
        """pack_row_from_block_launcher, bench_ghostserve_rdp.py:152-175."""
        _check_cuda(k_blk, v_blk, shards)
        if k_blk.element_size() != 2 or v_blk.element_size() != 2:
            raise ValueError("KV must be 16-bit words.")
        if shards.dim() != 2:
            raise ValueError("shards must be [rows, S].")
        words = k_blk.numel()
        p, pitch = _rows(shards, "shards")
        if shards.size(1) < 2 * words:
            raise ValueError("shard_size must be >= 2 * words.")
        _lib.call("gsec_rdpref_pack_row", _ptr(k_blk.contiguous()), _ptr(v_blk.contiguous()), words,
                  _lib.C.c_void_p(p), int(pitch), int(row), _s())

    @staticmethod
    def compute_rdp_parity(rows: torch.Tensor, nd: int, S: int, star_base: int) -> None:
        """compute_rdp_parity_launcher, bench_ghostserve_rdp.py:181-199."""
        _check_cuda(rows)
        if rows.dim() != 2 or rows.size(0) < nd + 2 or rows.size(1) < S:
            raise ValueError("bad shapes")
        p, pitch = _rows(rows, "rows")
        _lib.call("gsec_rdpref_parity", _lib.C.c_void_p(p), int(pitch), int(nd), int(S), int(star_base), _s())


xor_kernel = _XorKernel()
rdp_kernel = _RdpKernel()
rs_kernel = _RsKernel()
rdp_kv_ops = _RdpKvOps()
