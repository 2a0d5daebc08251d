"""Drop-in for the reference's benchmark/rdp/main.py: its mod-S row/diagonal
parity over the token-major u16 KV stream.

Same names, arguments, return structures and errors as the reference
(benchmark/rdp/main.py:21-126); parity and recovered bytes are the reference's
bit for bit.  Note on recovery: the reference's two-erasure path
(benchmark/rdp/kernel.cu:407-491) ends by rebuilding row min(a, b) from P with
every other row as it currently is and leaves the other row untouched, so it
only returns the original KV when the "missing" rows still hold their data (its
demo never erases them).  This module reproduces exactly that outcome; for real
double-failure recovery use the engine's textbook RDP (``codec.CodeSpec.rdp``).

Superset: bf16 KV is accepted (encoded as raw 16-bit words).  K and V are read
in their [B,H,T,D] layout and the token-major permutation is applied inside
the pack/unpack kernels instead of as separate .contiguous() copies.
"""
from __future__ import annotations

import argparse
import sys

import torch

if __package__ in (None, ""):  # run as a script (cd benchmark/rdp; python main.py ...), as the reference's demo is
    import importlib as _importlib
    import os as _os

    sys.path.insert(0, _os.path.dirname(_os.path.dirname(_os.path.dirname(_os.path.dirname(
        _os.path.abspath(__file__))))))
    __package__ = "26mlsys-ae-ghostserve_b200.benchmark.rdp"
    _importlib.import_module(__package__)

from ... import _lib  # noqa: E402
from ...codec import stream_handle  # noqa: E402


def _s():
    return _lib.C.c_void_p(stream_handle())


def determine_shard_size_words(total_words: int, num_data_shards: int):
    """benchmark/rdp/main.py:21-27."""
    if num_data_shards <= 0:
        raise ValueError("num_data_shards must be > 0")
    pad = (num_data_shards - (total_words % num_data_shards)) % num_data_shards
    padded_total = total_words + pad
    return padded_total // num_data_shards, pad


def fused_backup_full_kv(keys_bhtd: torch.Tensor, values_bhtd: torch.Tensor, num_data_shards: int,
                         star_base: int = 0):
    """benchmark/rdp/main.py:44-92: pack + P/Q parity in one call."""
    if not (keys_bhtd.is_cuda and values_bhtd.is_cuda):
        raise ValueError("keys/values must be CUDA tensors.")
    if keys_bhtd.dtype not in (torch.float16, torch.bfloat16) or values_bhtd.dtype != keys_bhtd.dtype:
        raise ValueError("keys/values must be fp16.")
    if keys_bhtd.shape != values_bhtd.shape:
        raise ValueError("K and V shapes must match [B,H,T,D].")
    if num_data_shards <= 0:
        raise ValueError("num_data_shards must be > 0")
    B, H, T, D = keys_bhtd.shape
    n = B * H * D
    total_words = 2 * T * n
    shard_size, pad_words = determine_shard_size_words(total_words, num_data_shards)
    nd = int(num_data_shards)
    pitch = -(-shard_size // 8) * 8
    buf = torch.empty((nd + 2, pitch), dtype=torch.uint16, device=keys_bhtd.device)
    k = keys_bhtd.contiguous()
    v = values_bhtd.contiguous()
    t0 = torch.cuda.Event(True)
    t1 = torch.cuda.Event(True)
    t0.record()
    _lib.call("gsec_rdpref_backup_bhtd", k.data_ptr(), v.data_ptr(), B, H, T, D, buf.data_ptr(), pitch, nd,
              shard_size, int(star_base), _s())
    t1.record()
    torch.cuda.synchronize()
    return {
        "shards_KV": buf[:, :shard_size],
        "shard_size": int(shard_size),
        "seq_len": int(T),
        "n": int(n),
        "num_data_shards": nd,
        "star_base": int(star_base),
        "shape_BHTD": (B, H, T, D),
        "backup_ms": t0.elapsed_time(t1),
        "pad_words": int(pad_words),
        "dtype": keys_bhtd.dtype,
    }


def fused_recovery_full_kv(pkg: dict, missing_a: int, missing_b: int = -1):
    """benchmark/rdp/main.py:95-126: recover and unpack to [B,H,T,D]."""
    shards = pkg["shards_KV"]
    shard_size = pkg["shard_size"]
    nd = pkg["num_data_shards"]
    star_base = pkg["star_base"]
    B, H, T, D = pkg["shape_BHTD"]
    dtype = pkg.get("dtype", torch.float16)
    if shards.dim() != 2 or shards.stride(1) != 1:
        raise ValueError("shards_KV must be [rows, S] with unit inner stride")
    keys = torch.empty((B, H, T, D), dtype=dtype, device=shards.device)
    values = torch.empty((B, H, T, D), dtype=dtype, device=shards.device)
    t0 = torch.cuda.Event(True)
    t1 = torch.cuda.Event(True)
    t0.record()
    _lib.call("gsec_rdpref_recovery_bhtd", shards.data_ptr(), shards.stride(0), keys.data_ptr(), values.data_ptr(),
              B, H, T, D, int(nd), int(shard_size), int(star_base), int(missing_a), int(missing_b), _s())
    t1.record()
    torch.cuda.synchronize()
    return keys, values, {"recover_ms": t0.elapsed_time(t1)}


def main(args):
    """The reference demo (benchmark/rdp/main.py:130-169) on this engine."""
    torch.manual_seed(0)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA required for this example.")
    device = torch.device("cuda")
    B, nh, T, hd = args.batch, args.heads, args.seq, args.head_dim
    print(f"Batch={B}, Heads={nh}, Seq={T}, HeadDim={hd}, N={B*nh*hd}")
    keys = torch.randn(B, nh, T, hd, device=device, dtype=torch.float16)
    values = torch.randn(B, nh, T, hd, device=device, dtype=torch.float16)
    ev = [torch.cuda.Event(True) for _ in range(4)]
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(5):
        pkg = fused_backup_full_kv(keys, values, args.num_data_shards, star_base=0)
    ev[1].record()
    ms = [m for m in args.missing_shards if m != -1]
    if len(ms) > 2:
        raise ValueError("RDP can only recover up to two missing data shards.")
    miss_a = ms[0] if len(ms) >= 1 else -1
    miss_b = ms[1] if len(ms) == 2 else -1
    torch.cuda.synchronize()
    ev[2].record()
    for _ in range(5):
        keys_q, values_q, _ = fused_recovery_full_kv(pkg, miss_a, miss_b)
    ev[3].record()
    torch.cuda.synchronize()
    print(f"total backup time: {ev[0].elapsed_time(ev[1])/5:.3f} ms")
    print(f"total recovery  time: {ev[2].elapsed_time(ev[3])/5:.3f} ms")


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description="Full-KV fp16-pack + RDP (parallel double-failure)")
    parser.add_argument("--num_data_shards", type=int, default=8)
    parser.add_argument("--missing_shards", type=int, nargs="*", default=[0, 1])
    parser.add_argument("--batch", type=int, default=1)
    parser.add_argument("--heads", type=int, default=8)
    parser.add_argument("--seq", type=int, default=512)
    parser.add_argument("--head_dim", type=int, default=128)
    args = parser.parse_args()
    if any((m != -1 and m >= args.num_data_shards) for m in args.missing_shards):
        print(f"Error: data shard indices must be -1 or in [0, {args.num_data_shards-1}].")
        sys.exit(1)
    main(args)
