"""numpy implementation of the engine's codes (TEST INFRASTRUCTURE ONLY).

The reference has no implementation of these two codes, so this module is the
builder's own restatement of the published algorithms, written independently
of the CUDA kernels:

* Row-Diagonal Parity, Corbett et al., "Row-Diagonal Parity for Double Disk
  Failure Correction", FAST 2004.  p prime, k <= p-1 data shards (missing data
  columns are all-zero: the shortened code), stripes of (p-1) units.
  Encoding: P = row XOR; Q[d] = XOR of the cells on diagonal d = (r + c) mod p
  over the data AND row-parity columns, diagonal p-1 not stored.
  Decoding here is by peeling: repeatedly solve any row or diagonal equation
  with exactly one unknown cell (the paper's chain recovery), which is a
  different procedure from the CUDA decoder's precomputed syndrome masks.
* Reed-Solomon over GF(2^8), polynomial x^8+x^4+x^3+x^2+1 (0x11d), generator
  [I_k ; C] with the Cauchy block C[j][i] = 1 / (x_j + y_i), x_j = k + j,
  y_i = i, "+" = XOR, no normalisation.  Decoding inverts the k x k matrix of
  the first k surviving rows by Gauss-Jordan elimination.
* XOR: single parity (the k+1 code of benchmark/xor without its byte layout).

Shards are 1-D ``np.uint8`` arrays.
"""
from __future__ import annotations

import numpy as np

# ============================================================= GF(2^8) 0x11d ==


def _gf8_tables():
    exp = np.zeros(512, dtype=np.uint8)
    log = np.zeros(256, dtype=np.int64)
    x = 1
    for i in range(255):
        exp[i] = x
        log[x] = i
        x <<= 1
        if x & 0x100:
            x ^= 0x11D
    exp[255:510] = exp[:255]
    return exp, log


GF8_EXP, GF8_LOG = _gf8_tables()


def gf8_mul(a, b):
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    r = GF8_EXP[(GF8_LOG[a] + GF8_LOG[b]) % 255]
    return np.where((a == 0) | (b == 0), 0, r).astype(np.uint8)


def gf8_inv(a: int) -> int:
    if a == 0:
        raise ZeroDivisionError("GF(2^8) inverse of 0")
    return int(GF8_EXP[(255 - GF8_LOG[a]) % 255])


def gf8_mul_bitwise(a: int, b: int) -> int:
    """Shift-and-add multiply (independent of the tables), for table checks."""
    r = 0
    for _ in range(8):
        if b & 1:
            r ^= a
        b >>= 1
        a <<= 1
        if a & 0x100:
            a ^= 0x11D
    return r


def rs8_generator(k: int, m: int) -> np.ndarray:
    g = np.zeros((k + m, k), dtype=np.uint8)
    g[:k] = np.eye(k, dtype=np.uint8)
    for j in range(m):
        for i in range(k):
            g[k + j, i] = gf8_inv((k + j) ^ i)
    return g


def _gf8_matvec(rows: np.ndarray, shards: list) -> list:
    out = []
    for row in rows:
        acc = np.zeros_like(shards[0])
        for c, s in zip(row, shards):
            if c:
                acc ^= gf8_mul(c, s)
        out.append(acc)
    return out


def gf8_invert(a: np.ndarray) -> np.ndarray:
    n = a.shape[0]
    a = a.astype(np.int64).copy()
    inv = np.eye(n, dtype=np.int64)
    for c in range(n):
        piv = next((r for r in range(c, n) if a[r, c]), None)
        if piv is None:
            raise ValueError("singular matrix")
        a[[c, piv]] = a[[piv, c]]
        inv[[c, piv]] = inv[[piv, c]]
        s = gf8_inv(int(a[c, c]))
        a[c] = gf8_mul(a[c], s)
        inv[c] = gf8_mul(inv[c], s)
        for r in range(n):
            if r != c and a[r, c]:
                f = int(a[r, c])
                a[r] ^= gf8_mul(f, a[c]).astype(np.int64)
                inv[r] ^= gf8_mul(f, inv[c]).astype(np.int64)
    return inv.astype(np.uint8)


def rs8_encode(data: list, m: int) -> list:
    k = len(data)
    return _gf8_matvec(rs8_generator(k, m)[k:], data)


def rs8_decode(shards: list, k: int, m: int) -> list:
    """shards: k+m entries, None where erased. Returns all k+m shards."""
    erased = [i for i, s in enumerate(shards) if s is None]
    if len(erased) > m:
        raise ValueError("too many erasures")
    if not erased:
        return list(shards)
    g = rs8_generator(k, m)
    surv = [i for i, s in enumerate(shards) if s is not None][:k]
    inv = gf8_invert(g[surv])
    data = _gf8_matvec(inv, [shards[i] for i in surv])
    out = list(shards)
    for i in erased:
        out[i] = data[i] if i < k else _gf8_matvec(g[i:i + 1], data)[0]
    return out


# ======================================================================== XOR ==


def xor_encode(data: list) -> np.ndarray:
    return np.bitwise_xor.reduce(np.stack(data), axis=0)


def xor_decode(shards: list) -> list:
    erased = [i for i, s in enumerate(shards) if s is None]
    if len(erased) > 1:
        raise ValueError("XOR rebuilds one shard")
    out = list(shards)
    if erased:
        out[erased[0]] = np.bitwise_xor.reduce(np.stack([s for s in shards if s is not None]), axis=0)
    return out


# ======================================================================== RDP ==


def rdp_parity_bytes(data_bytes: int, p: int, unit: int) -> int:
    sb = (p - 1) * unit
    return -(-data_bytes // sb) * sb


def _cells(shard: np.ndarray, nbytes: int, p: int, unit: int) -> np.ndarray:
    """Shard -> [stripes, p-1 rows, unit] (zero padded to whole stripes)."""
    buf = np.zeros(nbytes, dtype=np.uint8)
    buf[:shard.size] = shard
    return buf.reshape(-1, p - 1, unit)


def rdp_encode(data: list, p: int, unit: int):
    """Returns (P, Q) as 1-D arrays of rdp_parity_bytes(len(data[0])) bytes."""
    k = len(data)
    assert 1 <= k <= p - 1
    nbytes = rdp_parity_bytes(data[0].size, p, unit)
    cols = [_cells(d, nbytes, p, unit) for d in data]
    zero = np.zeros_like(cols[0])
    cols += [zero] * (p - 1 - k)          # virtual all-zero data columns
    P = np.bitwise_xor.reduce(np.stack(cols), axis=0)
    cols.append(P)                         # column p-1 takes part in the diagonals
    Q = np.zeros_like(P)
    for r in range(p - 1):
        for c in range(p):
            d = (r + c) % p
            if d != p - 1:
                Q[:, d] ^= cols[c][:, r]
    return P.reshape(-1), Q.reshape(-1)


def rdp_decode(shards: list, k: int, p: int, unit: int, data_bytes: int) -> list:
    """shards: k+2 entries (data..., P, Q), None where erased (at most two).
    Peeling decoder over the row and diagonal equations of each stripe."""
    erased = [i for i, s in enumerate(shards) if s is None]
    if len(erased) > 2:
        raise ValueError("RDP rebuilds at most two shards")
    nbytes = rdp_parity_bytes(data_bytes, p, unit)
    ns = nbytes // ((p - 1) * unit)
    col_of = {i: (i if i < k else (p - 1 if i == k else p)) for i in range(k + 2)}
    # cells[c][r]: known array [ns, unit] or None (unknown)
    cells = {}
    for c in range(p + 1):
        cells[c] = [np.zeros((ns, unit), dtype=np.uint8) for _ in range(p - 1)]
    for i, s in enumerate(shards):
        c = col_of[i]
        if s is None:
            cells[c] = [None] * (p - 1)
        else:
            arr = _cells(s, nbytes, p, unit)
            cells[c] = [arr[:, r] for r in range(p - 1)]
    eqs = []
    for r in range(p - 1):  # row r: columns 0..p-1 XOR to zero
        eqs.append([(c, r) for c in range(p)])
    for d in range(p - 1):  # diagonal d over columns 0..p-1, plus Q[d]
        eqs.append([(c, (d - c) % p) for c in range(p) if (d - c) % p != p - 1] + [(p, d)])
    progress = True
    while progress:
        progress = False
        for eq in eqs:
            unknown = [(c, r) for (c, r) in eq if cells[c][r] is None]
            if len(unknown) != 1:
                continue
            acc = np.zeros((ns, unit), dtype=np.uint8)
            for (c, r) in eq:
                if cells[c][r] is not None:
                    acc ^= cells[c][r]
            c, r = unknown[0]
            cells[c][r] = acc
            progress = True
    out = list(shards)
    for i in erased:
        c = col_of[i]
        if any(x is None for x in cells[c]):
            raise ValueError(f"erasure pattern {erased} not decodable")
        full = np.stack(cells[c], axis=1).reshape(-1)
        out[i] = full[:data_bytes].copy() if i < k else full.copy()
    return out
