"""Drop-in for the reference's benchmark/rs/main.py: Reed-Solomon over
GF(2^16) (polynomial 0x1100B, parity p coefficient alpha^((p+1)*i)) on the u16
stream [K | V].

Same names, arguments, return structures and errors as the reference
(benchmark/rs/main.py:39-206); parity and rebuilt data are the reference's
words exactly.  Differences:
* init_gf_tables() returns the same arrays, built in C instead of a Python loop;
  encode/decode do not need them (the library derives the same field).
* backwards_decode_kv also re-encodes erased parity rows (the reference leaves
  them zero) unless ``rebuild_parity=False``.
* bf16 KV is accepted as raw 16-bit words.
"""
from __future__ import annotations

import argparse
import sys

import numpy as np
import torch

if __package__ in (None, ""):  # run as a script (cd benchmark/rs; python main.py ...), as the reference's demo is
    import importlib as _importlib
    import os as _os

    sys.path.insert(0, _os.path.dirname(_os.path.dirname(_os.path.dirname(_os.path.dirname(
        _os.path.abspath(__file__))))))
    __package__ = "26mlsys-ae-ghostserve_b200.benchmark.rs"
    _importlib.import_module(__package__)

from ... import _lib  # noqa: E402
from ...codec import stream_handle  # noqa: E402

GF_SIZE = 1 << 16
GF_ORDER = GF_SIZE - 1


def _s():
    return _lib.C.c_void_p(stream_handle())


def init_gf_tables():
    """benchmark/rs/main.py:39-54 (same values)."""
    gf_exp = np.zeros(2 * GF_ORDER, dtype=np.uint16)
    gf_log = np.zeros(GF_SIZE, dtype=np.uint16)
    _lib.call("gsec_rs16_tables", gf_exp.ctypes.data, gf_log.ctypes.data)
    return gf_exp, gf_log


def shard_size_and_pad(total_symbols: int, num_data_shards: int):
    """benchmark/rs/main.py:57-60."""
    pad = (-total_symbols) % num_data_shards
    shard_size = (total_symbols + pad) // num_data_shards
    return shard_size, pad


def forward_encode_kv(keys: torch.Tensor, values: torch.Tensor, num_data_shards: int, num_parity_shards: int):
    """benchmark/rs/main.py:63-137. Returns (shards [k+m, shard_sz] u16, meta)."""
    assert keys.dtype in (torch.float16, torch.bfloat16) and values.dtype == keys.dtype
    device = keys.device
    assert device.type == "cuda"
    B, H, T, D = keys.shape
    N_k = keys.numel()
    N_v = values.numel()
    total = N_k + N_v
    assert total > 0, "Empty KV tensors"
    assert num_data_shards > 0 and num_parity_shards >= 0
    shard_sz, pad = shard_size_and_pad(total, num_data_shards)
    total_shards = num_data_shards + num_parity_shards
    assert shard_sz > 0
    pitch = -(-shard_sz // 8) * 8
    buf = torch.empty((total_shards, pitch), dtype=torch.uint16, device=device)
    k = keys.contiguous()
    v = values.contiguous()
    s = _s()
    _lib.call("gsec_rows_pack", k.data_ptr(), 2 * N_k, v.data_ptr(), 2 * N_v, buf.data_ptr(), 2 * pitch,
              2 * shard_sz, num_data_shards, s)
    _lib.call("gsec_rs16_encode", None, buf.data_ptr(), pitch, num_data_shards, num_parity_shards, shard_sz, s)
    meta = {
        "B": B, "H": H, "T": T, "D": D,
        "N_k": N_k, "N_v": N_v,
        "total": total,
        "pad": pad,
        "shard_sz": shard_sz,
        "num_data": num_data_shards,
        "num_parity": num_parity_shards,
        "dtype": keys.dtype,
    }
    return buf[:, :shard_sz], meta


def backwards_decode_kv(shards: torch.Tensor, meta: dict, missing_shards: list, rebuild_parity: bool = True):
    """benchmark/rs/main.py:140-206: rebuild missing data rows in place (from the
    first available parity rows, like the reference), then split into K, V."""
    device = shards.device
    num_data = meta["num_data"]
    num_parity = meta["num_parity"]
    shard_sz = meta["shard_sz"]
    dtype = meta.get("dtype", torch.float16)
    missing_data = sorted([i for i in missing_shards if i < num_data])
    missing_par = sorted([i - num_data for i in missing_shards if num_data <= i < num_data + num_parity])
    avail_par = [p for p in range(num_parity) if p not in missing_par]
    if len(missing_data) > len(avail_par):
        raise RuntimeError("Not enough parity shards to reconstruct the missing data shards.")
    if shards.dim() != 2 or shards.stride(1) != 1:
        raise ValueError("shards must be [rows, shard_sz] with unit inner stride")
    pitch = shards.stride(0)
    s = _s()
    if len(missing_data) > 0:
        if len(missing_data) > 16:
            raise RuntimeError("Reconstruction supports at most 16 missing data shards at once.")
        used = avail_par[:len(missing_data)]
        _lib.call("gsec_rs16_reconstruct", shards.data_ptr(), pitch, shard_sz, num_data, num_parity,
                  _lib.i32_array(missing_data), len(missing_data), _lib.i32_array(used), s)
    if rebuild_parity and missing_par:
        _lib.call("gsec_rs16_encode", None, shards.data_ptr(), pitch, num_data, num_parity, shard_sz, s)
    K = torch.empty(meta["N_k"], dtype=dtype, device=device)
    V = torch.empty(meta["N_v"], dtype=dtype, device=device)
    _lib.call("gsec_rows_unpack", shards.data_ptr(), 2 * pitch, 2 * shard_sz, num_data, K.data_ptr(),
              2 * meta["N_k"], V.data_ptr(), 2 * meta["N_v"], s)
    B, H, T, D = meta["B"], meta["H"], meta["T"], meta["D"]
    return K.view(B, H, T, D), V.view(B, H, T, D)


def main(num_data_shards: int, num_parity_shards: int, missing_shards: list, args):
    """The reference demo (benchmark/rs/main.py:209-248) on this engine."""
    torch.manual_seed(0)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA required.")
    device = torch.device("cuda")
    B, nh, T, hd = args.batch, args.heads, args.seq, args.head_dim
    keys = torch.randn(B, nh, T, hd, device=device, dtype=torch.float16)
    values = torch.randn_like(keys)
    ev = [torch.cuda.Event(True) for _ in range(4)]
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(5):
        shards, meta = forward_encode_kv(keys, values, num_data_shards, num_parity_shards)
    ev[1].record()
    shards_erase = shards.clone()
    for m in missing_shards:
        if 0 <= m < shards_erase.size(0):
            shards_erase[m].zero_()
        else:
            raise ValueError(f"Missing shard index {m} out of range 0..{shards_erase.size(0)-1}")
    torch.cuda.synchronize()
    ev[2].record()
    for _ in range(5):
        K_rec, V_rec = backwards_decode_kv(shards_erase, meta, missing_shards)
    ev[3].record()
    torch.cuda.synchronize()
    print(f"total backup time: {ev[0].elapsed_time(ev[1])/5:.3f} ms")
    print(f"total recovery  time: {ev[2].elapsed_time(ev[3])/5:.3f} ms")
    print(f"bit-exact: {torch.equal(K_rec.view(torch.int16), keys.view(torch.int16)) and torch.equal(V_rec.view(torch.int16), values.view(torch.int16))}")


if __name__ == "__main__":
    parser = argparse.ArgumentParser()
    parser.add_argument("--num_data_shards", type=int, default=8)
    parser.add_argument("--num_parity_shards", type=int, default=2)
    parser.add_argument("--missing_shards", type=int, nargs="+", default=[0, 1])
    parser.add_argument("--batch", type=int, default=1)
    parser.add_argument("--heads", type=int, default=8)
    parser.add_argument("--seq", type=int, default=256)
    parser.add_argument("--head_dim", type=int, default=128)
    args = parser.parse_args()
    if len(args.missing_shards) > (args.num_data_shards + args.num_parity_shards):
        print("Error: Too many missing shards!")
        sys.exit(1)
    main(args.num_data_shards, args.num_parity_shards, args.missing_shards, args)
