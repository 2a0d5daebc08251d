"""Drop-in for the reference's benchmark/xor/main.py: single-parity XOR of the
KV byte stream [K bytes | V bytes], split into k data shards plus one parity.

Same function names, arguments, return structures and errors as the
reference (benchmark/xor/main.py:39-212).  Superset: K/V may be any dtype (the
bytes are encoded as they lie in memory, so fp16 gives the reference's bytes,
bf16/fp8 KV are encoded raw instead of being rejected).

The shard buffer is allocated with rows padded to 16 bytes and returned as a
[k+1, shard_size] view, so the kernels take their vector path for every k;
decode accepts that view or any [k+1, shard_size] tensor with unit inner stride.
"""
from __future__ import annotations

import argparse
import sys

import torch

if __package__ in (None, ""):  # run as a script (cd benchmark/xor; python main.py ...), as the reference's demo is
    import importlib as _importlib
    import os as _os

    sys.path.insert(0, _os.path.dirname(_os.path.dirname(_os.path.dirname(_os.path.dirname(
        _os.path.abspath(__file__))))))
    __package__ = "26mlsys-ae-ghostserve_b200.benchmark.xor"
    _importlib.import_module(__package__)

from ... import _lib  # noqa: E402
from ...codec import stream_handle  # noqa: E402


def _s():
    return _lib.C.c_void_p(stream_handle())


def determine_shard_size(num_bytes: int, num_data_shards: int):
    """benchmark/xor/main.py:39-43."""
    pad = (num_data_shards - (num_bytes % num_data_shards)) % num_data_shards
    padded_total = num_bytes + pad
    shard_size = padded_total // num_data_shards
    return shard_size, pad


def forward_encode_kv(keys, values, num_data_shards, num_parity_shards):
    """benchmark/xor/main.py:47-133: pack [K|V] bytes, pad to k shards, encode.

    One kernel writes the padded data rows straight from K and V (the
    reference's pack, zero-pad copy and data copy) and one computes parity."""
    if num_parity_shards != 1:
        raise ValueError("XOR parity supports exactly 1 parity shard.")
    assert keys.is_cuda and values.is_cuda, "Run on CUDA for GPU timing."
    assert keys.dtype == values.dtype
    assert keys.shape == values.shape
    keys = keys.contiguous()
    values = values.contiguous()
    device = keys.device
    B, H, T, D = keys.shape
    n = B * H * D
    esz = keys.element_size()
    half = T * n * esz
    total_bytes = 2 * half  # 4*T*n for fp16, as in the reference

    shard_size, pad = determine_shard_size(total_bytes, num_data_shards)
    data_bytes = num_data_shards * shard_size
    total_shards = num_data_shards + num_parity_shards
    pitch = -(-shard_size // 16) * 16
    buf = torch.empty((total_shards, pitch), dtype=torch.uint8, device=device)
    s = _s()
    _lib.call("gsec_rows_pack", keys.data_ptr(), half, values.data_ptr(), half, buf.data_ptr(), pitch, shard_size,
              num_data_shards, s)
    _lib.call("gsec_xor_encode", None, buf.data_ptr(), num_data_shards, shard_size, pitch, s)
    shards_KV = buf[:, :shard_size]

    pack_io = 4 * T * n + total_bytes
    encode_io = data_bytes + data_bytes + shard_size
    return {
        "shards_KV": shards_KV,
        "seq_len": T,
        "n": n,
        "shard_size": shard_size,
        "device": device,
        "shape_BHTD": (B, H, T, D),
        "pack_io": pack_io,
        "encode_io": encode_io,
        "num_data_shards": num_data_shards,
        "num_parity_shards": num_parity_shards,
        "pad": pad,
        "total_bytes": total_bytes,
        "orig_keys": keys,
        "orig_vals": values,
    }


def backwards_decode_kv(pkg, missing_shards):
    """benchmark/xor/main.py:137-212: zero the missing shard, rebuild it in
    place, unpack back to K, V (bit-exact)."""
    shards_KV = pkg["shards_KV"]
    T = pkg["seq_len"]
    n = pkg["n"]
    shard_size = pkg["shard_size"]
    device = pkg["device"]
    B, H, _, D = pkg["shape_BHTD"]
    num_data_shards = pkg["num_data_shards"]
    num_parity_shards = pkg["num_parity_shards"]
    total_shards = num_data_shards + num_parity_shards
    dtype = pkg["orig_keys"].dtype if "orig_keys" in pkg else torch.float16

    if num_parity_shards != 1:
        raise ValueError("XOR parity supports exactly 1 parity shard.")
    if len(missing_shards) > 1:
        raise ValueError("XOR parity can recover only a single missing shard.")
    for idx in missing_shards:
        if idx < 0 or idx >= total_shards:
            raise ValueError(f"Missing shard {idx} out of range 0..{total_shards-1}")
    if shards_KV.dim() != 2 or shards_KV.stride(1) != 1:
        raise ValueError("shards_KV must be [shards, shard_size] with unit inner stride")
    for idx in missing_shards:
        shards_KV[idx].zero_()

    r_ms = 0.0
    pitch = shards_KV.stride(0)
    s = _s()
    if len(missing_shards) == 1:
        recovered_missing = torch.empty((1, shard_size), dtype=torch.uint8, device=device)
        _lib.call("gsec_xor_reconstruct", shards_KV.data_ptr(), recovered_missing.data_ptr(), shard_size, pitch,
                  num_data_shards, _lib.i32_array(missing_shards), 1, s)

    esz = torch.empty((), dtype=dtype).element_size()
    de_bytes_needed = 2 * T * n * esz
    if num_data_shards * shard_size < de_bytes_needed:
        raise RuntimeError("Not enough bytes in reconstructed data region.")
    dequant_KV = torch.empty(2 * T * n, dtype=dtype, device=device)
    _lib.call("gsec_rows_unpack", shards_KV.data_ptr(), pitch, shard_size, num_data_shards, dequant_KV.data_ptr(),
              de_bytes_needed, None, 0, s)

    de_io = de_bytes_needed + 4 * T * n
    keys_out = dequant_KV[:T * n].view(B, H, T, D)
    values_out = dequant_KV[T * n: 2 * T * n].view(B, H, T, D)
    return keys_out, values_out, {
        "reconstruct_ms": r_ms,
        "reconstruct_io": ((num_data_shards + 1) * shard_size + 2 * shard_size) if r_ms > 0 else 0,
        "unpack_io": de_io,
    }


def run(args):
    """The reference demo (benchmark/xor/main.py:216-254) on this engine."""
    torch.manual_seed(0)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA required for this example.")
    device = torch.device("cuda")
    B, nh, T, hd = args.batch, args.heads, args.seq, args.head_dim
    keys = torch.randn(B, nh, T, hd, device=device, dtype=torch.float16).contiguous()
    values = torch.randn(B, nh, T, hd, device=device, dtype=torch.float16).contiguous()
    print(f'Batch={B}, Heads={nh}, Seq={T}, HeadDim={hd}, N={B*nh*hd}')
    t = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    t[0].record()
    for _ in range(5):
        pkg = forward_encode_kv(keys, values, args.num_data_shards, args.num_parity_shards)
    t[1].record()
    torch.cuda.synchronize()
    t[2].record()
    for _ in range(5):
        keys_rt, values_rt, _ = backwards_decode_kv(pkg, args.missing_shards)
    t[3].record()
    torch.cuda.synchronize()
    print(f"total backup time: {t[0].elapsed_time(t[1]):.3f} ms")
    print(f"total recovery  time: {t[2].elapsed_time(t[3]):.3f} ms")
    print(f"bit-exact: {torch.equal(keys.view(torch.int16), keys_rt.view(torch.int16)) and torch.equal(values.view(torch.int16), values_rt.view(torch.int16))}")


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--num_data_shards", type=int, default=8)
    parser.add_argument("--num_parity_shards", type=int, default=1)
    parser.add_argument("--missing_shards", type=int, nargs="+", default=[3])
    parser.add_argument("--batch", type=int, default=1)
    parser.add_argument("--heads", type=int, default=8)
    parser.add_argument("--seq", type=int, default=256)
    parser.add_argument("--head_dim", type=int, default=128)
    args = parser.parse_args()
    total = args.num_data_shards + args.num_parity_shards
    if args.num_parity_shards != 1:
        print("Error: XOR parity supports exactly 1 parity shard.")
        sys.exit(1)
    if len(args.missing_shards) > 1:
        print("Error: XOR parity can only recover a single missing shard.")
        sys.exit(1)
    if any((m < 0 or m >= total) for m in args.missing_shards):
        print(f"Error: missing shard index must be in [0, {total-1}].")
        sys.exit(1)
    run(args)


if __name__ == "__main__":
    main()
