"""Known-answer vectors for the engine's codes, from a second restatement of the
published algorithms that shares no code or table with ``oracle/codes.py``.

    python tests/golden/kat.py          # rewrites tests/golden/kat_codes.json (CPU only)

TEST INFRASTRUCTURE. The reference project has no implementation of the two
codes the benchmark configs measure (textbook RDP for config 1, RS(6,2) over
GF(2^8) for config 2), so nothing of the reference can pin them. This file
pins them a second way:

* GF(2^8) with polynomial x^8+x^4+x^3+x^2+1 (0x11d) by shift-and-add
  multiplication only; inverses by exhaustive search; the Cauchy block
  C[j][i] = 1 / ((k + j) XOR i) built from those.
* Row-Diagonal Parity (Corbett et al., FAST 2004, section 3) encoded by
  walking each diagonal: diagonal d takes, for each disk j in 0..p-1 (data
  disks 0..p-2, row-parity disk p-1), the block in row (d - j) mod p, unless
  that row is p-1 (the diagonal misses disk j). The oracle instead scatters
  every cell into diagonal (r + c) mod p.

Inputs are drawn from numpy's seeded generator (bf16 bit patterns of N(0,1)
floats, or uniform bytes), so the same bytes can be rebuilt anywhere from the
seed. ``kat_codes.json`` stores, per case, the SHA-256 of every parity shard
(and the first bytes in hex for a readable diff); the GPU tests and
``bench.py`` rebuild the inputs, run the CUDA encode and compare hashes.
"""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KAT_FILE = os.path.join(HERE, "kat_codes.json")
MIB = 1 << 20


# ------------------------------------------------------------------ inputs ---
def shard_bytes(kind: str, seed: int, j: int, nbytes: int) -> np.ndarray:
    """Data shard j of a case: ``nbytes`` bytes, a pure function of (seed, j).
    kind "bf16": bf16 bit patterns of float32 N(0,1) draws (truncation);
    kind "u8": uniform random bytes (the fp8 KV configs)."""
    rng = np.random.default_rng([seed, j])
    if kind == "bf16":
        x = rng.standard_normal(nbytes // 2, dtype=np.float32)
        return (x.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8)
    return rng.integers(0, 256, nbytes, dtype=np.uint8)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).view(np.uint8).tobytes()).hexdigest()


# ---------------------------------------------------------------- GF(2^8) ---
POLY = 0x11D


def gf_mul(a: int, b: int) -> int:
    """Shift-and-add product in GF(2^8)/0x11d."""
    acc = 0
    while b:
        if b & 1:
            acc ^= a
        a <<= 1
        if a & 0x100:
            a ^= POLY
        b >>= 1
    return acc


def gf_inv(a: int) -> int:
    """Exhaustive search for the b with a*b = 1."""
    for b in range(1, 256):
        if gf_mul(a, b) == 1:
            return b
    raise ZeroDivisionError(a)


def cauchy(k: int, m: int) -> list:
    """m x k Cauchy block: C[j][i] = 1 / ((k + j) XOR i)."""
    return [[gf_inv((k + j) ^ i) for i in range(k)] for j in range(m)]


def rs8_encode(data: list, m: int) -> list:
    """Parity shard j = sum_i C[j][i] * D_i, byte by byte (products from a
    256-entry row of gf_mul per coefficient)."""
    k = len(data)
    out = []
    for row in cauchy(k, m):
        acc = np.zeros_like(data[0])
        for c, d in zip(row, data):
            table = np.array([gf_mul(c, b) for b in range(256)], dtype=np.uint8)
            acc ^= table[d]
        out.append(acc)
    return out


# --------------------------------------------------------------------- RDP ---
def rdp_encode(data: list, p: int, unit: int):
    """(P, Q) of textbook RDP(p) over k <= p-1 data shards (shards k..p-2 are
    all-zero), stripes of p-1 units of ``unit`` bytes, shards zero-padded to
    whole stripes. Q is computed by walking each diagonal across the disks."""
    rows = p - 1
    nbytes = len(data[0])
    sb = rows * unit
    stripes = -(-nbytes // sb)
    disk = []  # disk j as [stripes, rows, unit]
    for j in range(p - 1):
        buf = np.zeros(stripes * sb, dtype=np.uint8)
        if j < len(data):
            buf[:nbytes] = data[j]
        disk.append(buf.reshape(stripes, rows, unit))
    P = np.zeros((stripes, rows, unit), dtype=np.uint8)
    for j in range(p - 1):
        P ^= disk[j]
    disk.append(P)  # disk p-1: row parity
    Q = np.zeros((stripes, rows, unit), dtype=np.uint8)
    for d in range(p - 1):
        for j in range(p):
            i = (d - j) % p
            if i != p - 1:
                Q[:, d, :] ^= disk[j][:, i, :]
    return P.reshape(-1), Q.reshape(-1)


def xor_encode(data: list) -> np.ndarray:
    acc = np.zeros_like(data[0])
    for d in data:
        acc ^= d
    return acc


# ------------------------------------------------------------------- cases ---
# (name, scheme, k, m, p, unit, kind, shard bytes, seed). The first three are the
# benchmark's configs 0-2 at full size; the rest are small and ragged (partial
# tail stripes, shortened RDP, every RS8 parity count the engine supports).
CASES = [
    ("config0_xor_7", "xor", 7, 1, 0, 0, "bf16", 32 * MIB, 100),
    ("config1_rdp_p7", "rdp", 6, 2, 7, 4096, "bf16", 32 * MIB, 101),
    ("config2_rs8_6_2", "rs8", 6, 2, 0, 0, "u8", 16 * MIB, 102),
    ("rdp_p3_k2_tail", "rdp", 2, 2, 3, 1024, "bf16", 5 * 2048 + 1024 + 16, 103),
    ("rdp_p5_k3_short", "rdp", 3, 2, 5, 2048, "u8", 3 * 8192 + 4096, 104),
    ("rdp_p7_k6_unit16", "rdp", 6, 2, 7, 16, "u8", 96 * 7 + 32, 105),
    ("rdp_p11_k8", "rdp", 8, 2, 11, 1024, "bf16", 2 * 10240 + 512, 106),
    ("rs8_2_1", "rs8", 2, 1, 0, 0, "u8", 4096 + 48, 107),
    ("rs8_4_3", "rs8", 4, 3, 0, 0, "u8", 8192, 108),
    ("rs8_6_4", "rs8", 6, 4, 0, 0, "bf16", 65536 + 16, 109),
    ("xor_1", "xor", 1, 1, 0, 0, "u8", 4096, 110),
]


def case_data(case) -> list:
    name, scheme, k, m, p, unit, kind, nbytes, seed = case
    return [shard_bytes(kind, seed, j, nbytes) for j in range(k)]


def case_parity(case, data=None) -> list:
    name, scheme, k, m, p, unit, kind, nbytes, seed = case
    data = case_data(case) if data is None else data
    if scheme == "rdp":
        return list(rdp_encode(data, p, unit))
    if scheme == "rs8":
        return rs8_encode(data, m)
    return [xor_encode(data)]


def main() -> None:
    out = {"generator": "tests/golden/kat.py", "poly": "0x11d",
           "cauchy_6_2": cauchy(6, 2), "cases": {}}
    for case in CASES:
        name, scheme, k, m, p, unit, kind, nbytes, seed = case
        par = case_parity(case)
        out["cases"][name] = {
            "scheme": scheme, "k": k, "m": m, "p": p, "unit": unit, "kind": kind, "shard_bytes": nbytes,
            "seed": seed, "parity_bytes": int(par[0].size),
            "parity_sha256": [sha(x) for x in par], "parity_head_hex": [x[:16].tobytes().hex() for x in par]}
    with open(KAT_FILE, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
