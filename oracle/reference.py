"""numpy restatement of the reference's erasure codes (TEST INFRASTRUCTURE ONLY).

Every function follows one reference function and cites it.  KV tensors are
handled as their raw 16-bit patterns (``np.uint16``), which is exactly what the
reference kernels operate on (they reinterpret fp16 as uint16 or bytes).
Paths are relative to the reference project root.
"""
from __future__ import annotations

import numpy as np

GF16_SIZE = 1 << 16
GF16_ORDER = GF16_SIZE - 1

# ============================================================================ XOR
# benchmark/xor


def determine_shard_size(num_bytes: int, num_data_shards: int):
    """benchmark/xor/main.py:39-43."""
    pad = (num_data_shards - (num_bytes % num_data_shards)) % num_data_shards
    padded_total = num_bytes + pad
    return padded_total // num_data_shards, pad


def xor_pack_kv(keys: np.ndarray, values: np.ndarray) -> np.ndarray:
    """pack_kv_kernel, benchmark/xor/kernel.cu:93-119: [K bytes | V bytes], each
    half little-endian (low byte first) in flattening order."""
    k = np.ascontiguousarray(keys, dtype=np.uint16).reshape(-1)
    v = np.ascontiguousarray(values, dtype=np.uint16).reshape(-1)
    out = np.empty(4 * k.size, dtype=np.uint8)
    out[0:2 * k.size:2] = k & 0xFF
    out[1:2 * k.size:2] = k >> 8
    out[2 * k.size::2] = v & 0xFF
    out[2 * k.size + 1::2] = v >> 8
    return out


def xor_unpack_kv(kv_bytes: np.ndarray, total: int) -> np.ndarray:
    """unpack_kv_kernel, benchmark/xor/kernel.cu:122-146: returns [K | V] as u16."""
    b = kv_bytes[:4 * total].astype(np.uint16)
    return (b[0::2] | (b[1::2] << 8)).astype(np.uint16)


def xor_encode(data_padded: np.ndarray, data_shards: int, shard_size: int) -> np.ndarray:
    """encode_xor_kernel, benchmark/xor/kernel.cu:17-41: rows 0..k-1 copy the data,
    row k is the byte-wise XOR."""
    d = data_padded[:data_shards * shard_size].reshape(data_shards, shard_size)
    shards = np.zeros((data_shards + 1, shard_size), dtype=np.uint8)
    shards[:data_shards] = d
    shards[data_shards] = np.bitwise_xor.reduce(d, axis=0)
    return shards


def xor_reconstruct(shards: np.ndarray, shard_size: int, data_shards: int, missing: list):
    """reconstruct_xor_kernel, benchmark/xor/kernel.cu:47-88, called in place as in
    benchmark/xor/main.py:174-177. Returns (shards, recovered_missing or None)."""
    if len(missing) != 1:
        return shards, None
    m = missing[0]
    if 0 <= m < data_shards:
        acc = shards[data_shards].copy()
        for k in range(data_shards):
            if k != m:
                acc ^= shards[k]
        shards[m] = acc
        return shards, acc.copy()
    if m == data_shards:
        acc = np.bitwise_xor.reduce(shards[:data_shards], axis=0)
        shards[data_shards] = acc
        return shards, acc.copy()
    return shards, None


def xor_forward_encode_kv(keys: np.ndarray, values: np.ndarray, num_data_shards: int):
    """forward_encode_kv, benchmark/xor/main.py:47-133 (byte work only)."""
    kv = xor_pack_kv(keys, values)
    shard_size, pad = determine_shard_size(kv.size, num_data_shards)
    data_padded = np.zeros(num_data_shards * shard_size, dtype=np.uint8)
    data_padded[:kv.size] = kv
    return xor_encode(data_padded, num_data_shards, shard_size), shard_size, pad


def xor_backwards_decode_kv(shards: np.ndarray, shape_bhtd, num_data_shards: int, missing: list):
    """backwards_decode_kv, benchmark/xor/main.py:137-212: zero the missing shard,
    rebuild it, unpack. Returns (keys_u16, values_u16, shards)."""
    shards = shards.copy()
    shard_size = shards.shape[1]
    for idx in missing:
        shards[idx] = 0
    if len(missing) == 1:
        xor_reconstruct(shards, shard_size, num_data_shards, missing)
    total = int(np.prod(shape_bhtd))
    kv = xor_unpack_kv(shards[:num_data_shards].reshape(-1), total)
    return kv[:total].reshape(shape_bhtd), kv[total:2 * total].reshape(shape_bhtd), shards


# ====================================================================== RDP-ref
# benchmark/rdp and bench_ghostserve_rdp.py:92-207


def determine_shard_size_words(total_words: int, num_data_shards: int):
    """benchmark/rdp/main.py:21-27."""
    if num_data_shards <= 0:
        raise ValueError("num_data_shards must be > 0")
    pad = (num_data_shards - (total_words % num_data_shards)) % num_data_shards
    return (total_words + pad) // num_data_shards, pad


def to_tn(x_bhtd: np.ndarray) -> np.ndarray:
    """[B,H,T,D] -> [T, B*H*D], benchmark/rdp/main.py:66-67."""
    B, H, T, D = x_bhtd.shape
    return np.ascontiguousarray(x_bhtd.transpose(2, 0, 1, 3)).reshape(T, B * H * D)


def from_tn(x_tn: np.ndarray, shape_bhtd) -> np.ndarray:
    """[T, n] -> [B,H,T,D], benchmark/rdp/main.py:121-124."""
    B, H, T, D = shape_bhtd
    return np.ascontiguousarray(x_tn.reshape(T, B, H, D).transpose(1, 2, 0, 3))


def rdpref_pack(k_tn: np.ndarray, v_tn: np.ndarray, nd: int, S: int) -> np.ndarray:
    """pack_scatter_kernel_full, benchmark/rdp/kernel.cu:32-72, into the zeroed
    shards of benchmark/rdp/main.py:73: stream [K_TN | V_TN] cut into rows of S."""
    stream = np.concatenate([k_tn.reshape(-1), v_tn.reshape(-1)]).astype(np.uint16)
    shards = np.zeros((nd + 2, S), dtype=np.uint16)
    flat = shards[:nd].reshape(-1)
    flat[:stream.size] = stream
    shards[:nd] = flat.reshape(nd, S)
    return shards


def c_mod(a: int, b: int) -> int:
    """C/C++ integer remainder (truncates toward zero)."""
    r = abs(a) % abs(b)
    return -r if a < 0 else r


def star_exclusions(nd: int, S: int, star_base: int) -> np.ndarray:
    """Q position whose row-r term is skipped: (d - r) mod S == star_r with
    star_r = (star_base + r) % S (C remainder), benchmark/rdp/kernel.cu:100-102;
    -1 when star_r is negative (never equals a non-negative column)."""
    out = np.full(nd, -1, dtype=np.int64)
    for r in range(nd):
        sr = c_mod(star_base + r, S)
        if sr >= 0:
            out[r] = (sr + r) % S
    return out


def rdpref_parity(shards: np.ndarray, nd: int, S: int, star_base: int) -> np.ndarray:
    """compute_rdp_parity_kernel, benchmark/rdp/kernel.cu:76-107 (same math as the
    hook's kernel, bench_ghostserve_rdp.py:121-150). Writes rows nd (P), nd+1 (Q)."""
    d = shards[:nd]
    shards[nd] = np.bitwise_xor.reduce(d, axis=0)
    q = np.zeros(S, dtype=np.uint16)
    ex = star_exclusions(nd, S, star_base)
    for r in range(nd):
        term = np.roll(d[r], r)  # term[dd] = D[r][(dd - r) mod S]
        if ex[r] >= 0:
            term = term.copy()
            term[ex[r]] = 0
        q ^= term
    shards[nd + 1] = q
    return shards


def rdpref_reconstruct_single(shards: np.ndarray, nd: int, S: int, miss: int) -> np.ndarray:
    """rdp_reconstruct_single_kernel, benchmark/rdp/kernel.cu:111-128."""
    if nd <= 0 or S <= 0 or miss < 0 or miss >= nd:
        return shards
    acc = shards[nd].copy()
    for r in range(nd):
        if r != miss:
            acc ^= shards[r]
    shards[miss] = acc
    return shards


def _rebuild_row_from_p(shards, nd, S, target):
    """rebuild_row_from_P, benchmark/rdp/kernel.cu:286-301."""
    acc = shards[nd].copy()
    for r in range(nd):
        if r != target:
            acc ^= shards[r]
    shards[target] = acc


def _blelloch_exclusive_xor(w: np.ndarray, threads: int = 256) -> np.ndarray:
    """The in-tile scan of rdp_double_tile_provisional_A_only,
    benchmark/rdp/kernel.cu:198-217, step for step (exact for power-of-two tiles,
    what the kernel computes otherwise)."""
    px = w.copy()
    n = px.size
    tids = np.arange(threads)
    offset = 1
    while offset < n:
        idx = (tids + 1) * (offset << 1) - 1
        idx = idx[idx < n]
        px[idx] ^= px[idx - offset]
        offset <<= 1
    px[n - 1] = 0
    offset = n >> 1
    while offset > 0:
        idx = (tids + 1) * (offset << 1) - 1
        idx = idx[idx < n]
        t = px[idx - offset].copy()
        px[idx - offset] = px[idx]
        px[idx] ^= t
        offset >>= 1
    return px


def rdpref_recovery(shards: np.ndarray, nd: int, S: int, star_base: int, miss_a: int, miss_b: int,
                    tile_k: int = 256) -> np.ndarray:
    """fused_recovery_full_kv_launcher's recovery half, benchmark/rdp/kernel.cu:397-507,
    every step restated in order (provisional ring solve per tile, host carry scan,
    carry apply, star fill, then rebuild_row_from_P(a) and rebuild_row_from_P(b))."""
    def norm(m):
        return m if 0 <= m < nd else -1

    a, b = norm(miss_a), norm(miss_b)
    if a >= 0 and b >= 0 and a != b:
        if b < a:
            a, b = b, a
        star_b = c_mod(star_base + b, S)
        delta = (b - a) % S
        d_b = (star_b + b) % S
        pos0 = (d_b - a) % S
        L = S - 1 if S > 0 else 0
        num_tiles = (L + tile_k - 1) // tile_k
        star_a = c_mod(star_base + a, S)
        ex = star_exclusions(nd, S, star_base)
        others = [r for r in range(nd) if r not in (a, b)]
        carries = np.zeros(max(1, num_tiles), dtype=np.uint16)
        for tile in range(num_tiles):
            k0 = tile * tile_k
            tl = min(tile_k, L - k0)
            pos = (pos0 + (k0 % S) * delta) % S
            pos_j = (pos + np.arange(tl, dtype=np.int64) * delta) % S
            d_a = (pos_j + a) % S
            rp = shards[nd][pos_j].copy()  # rhs_rowP_except_ab, :132-141
            for r in others:
                rp ^= shards[r][pos_j]
            rq = shards[nd + 1][d_a].copy()  # rhs_diagQ_except_ab, :143-155
            for r in others:
                c = (d_a - r) % S
                term = shards[r][c]
                if ex[r] >= 0:
                    term = np.where(d_a == ex[r], np.uint16(0), term)
                rq ^= term
            w = rp ^ rq
            px = _blelloch_exclusive_xor(w)
            keep = pos_j != star_a
            shards[a][pos_j[keep]] = (rq ^ px)[keep]
            carries[tile] = np.bitwise_xor.reduce(w) if w.size else 0
        acc = np.uint16(0)  # exclusive prefix on the host, :439-449
        tin = np.zeros_like(carries)
        for i in range(num_tiles):
            tin[i] = acc
            acc ^= carries[i]
        for tile in range(num_tiles):  # rdp_double_tile_fix_apply_A, :244-264
            k0 = tile * tile_k
            tl = min(tile_k, L - k0)
            pos = (pos0 + (k0 % S) * delta) % S
            for j in range(tl):
                pj = (pos + j * delta) % S
                shards[a][pj] ^= tin[tile]
        if star_a >= 0:  # fill_a_star_from_P, :268-282
            accs = shards[nd][star_a]
            for r in range(nd):
                if r != a:
                    accs ^= shards[r][star_a]
            shards[a][star_a] = accs
        _rebuild_row_from_p(shards, nd, S, a)  # :472-480
        _rebuild_row_from_p(shards, nd, S, b)  # :482-490
    elif a >= 0 and b < 0:
        rdpref_reconstruct_single(shards, nd, S, a)
    elif b >= 0 and a < 0:
        rdpref_reconstruct_single(shards, nd, S, b)
    return shards


def rdpref_recovery_outcome(shards: np.ndarray, nd: int, miss_a: int, miss_b: int) -> np.ndarray:
    """Closed form of rdpref_recovery: the only surviving effect of the whole
    sequence is that row min(a, b) (or the single valid index) becomes
    P ^ XOR(all other data rows as they currently are)."""
    def norm(m):
        return m if 0 <= m < nd else -1

    a, b = norm(miss_a), norm(miss_b)
    if a >= 0 and b >= 0:
        target = min(a, b) if a != b else -1
    else:
        target = a if a >= 0 else b
    if target >= 0:
        _rebuild_row_from_p(shards, nd, shards.shape[1], target)
    return shards


def rdpref_load_full(shards: np.ndarray, T: int, n: int, nd: int, S: int) -> np.ndarray:
    """load_full_kernel, benchmark/rdp/kernel.cu:305-345: rows -> [K_TN | V_TN]."""
    flat = shards[:nd].reshape(-1)
    out = np.zeros(2 * T * n, dtype=np.uint16)
    m = min(out.size, flat.size)
    out[:m] = flat[:m]
    return out


def rdpref_backup(keys: np.ndarray, values: np.ndarray, nd: int, star_base: int = 0):
    """fused_backup_full_kv, benchmark/rdp/main.py:44-92 (byte work). Returns
    (shards, S, pad_words)."""
    B, H, T, D = keys.shape
    n = B * H * D
    S, pad = determine_shard_size_words(2 * T * n, nd)
    shards = rdpref_pack(to_tn(keys), to_tn(values), nd, S)
    rdpref_parity(shards, nd, S, star_base)
    return shards, S, pad


# ------------------------------------------------------------------ the hook --


def hook_pack_row(k_blk: np.ndarray, v_blk: np.ndarray, rows: np.ndarray, row: int) -> None:
    """pack_row_from_block_kernel, bench_ghostserve_rdp.py:105-118."""
    w = k_blk.size
    rows[row, :w] = k_blk.reshape(-1)
    rows[row, w:2 * w] = v_blk.reshape(-1)


def hook_compute_parity(k_all_u16: np.ndarray, v_all_u16: np.ndarray, elems: int, star_base: int = 0):
    """_compute_parity_to_cpu, bench_ghostserve_rdp.py:334-367, for inputs that are
    already the fp16 bit patterns the hook packs (it value-casts with
    .to(torch.float16) first, :345-346). Returns (P, Q) as u16 rows."""
    world = k_all_u16.size // elems
    S = 2 * elems
    rows = np.zeros((world + 2, S), dtype=np.uint16)
    for r in range(world):
        hook_pack_row(k_all_u16[r * elems:(r + 1) * elems], v_all_u16[r * elems:(r + 1) * elems], rows, r)
    rdpref_parity(rows, world, S, star_base)
    return rows[world].copy(), rows[world + 1].copy()


# ========================================================================= RS16
# benchmark/rs


def init_gf_tables():
    """benchmark/rs/main.py:39-54: exp (2*65535) and log (65536), poly 0x1100B."""
    primitive_polynomial = 0x1100B
    gf_log = np.zeros(GF16_SIZE, dtype=np.uint16)
    gf_exp = np.zeros(2 * GF16_ORDER, dtype=np.uint16)
    x = 1
    for i in range(GF16_ORDER):
        gf_exp[i] = x
        gf_log[x] = i
        x <<= 1
        if x & GF16_SIZE:
            x ^= primitive_polynomial
    gf_exp[GF16_ORDER:] = gf_exp[:GF16_ORDER]
    return gf_exp, gf_log


_TABLES = None


def gf16_tables():
    global _TABLES
    if _TABLES is None:
        _TABLES = init_gf_tables()
    return _TABLES


def gf16_mul(a, b):
    """gf_mul, benchmark/rs/kernel.cu:16-23 (vectorised)."""
    exp, log = gf16_tables()
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    s = log[a].astype(np.int64) + log[b].astype(np.int64)
    s = np.where(s >= GF16_ORDER, s - GF16_ORDER, s)
    return np.where((a == 0) | (b == 0), 0, exp[s]).astype(np.uint16)


def gf16_div(a: int, b: int) -> int:
    """gf_div, benchmark/rs/kernel.cu:25-33."""
    exp, log = gf16_tables()
    if a == 0 or b == 0:
        return 0
    d = int(log[a]) - int(log[b])
    if d < 0:
        d += GF16_ORDER
    return int(exp[d])


def shard_size_and_pad(total_symbols: int, num_data_shards: int):
    """benchmark/rs/main.py:57-60."""
    pad = (-total_symbols) % num_data_shards
    return (total_symbols + pad) // num_data_shards, pad


def rs16_encode(data_padded: np.ndarray, data_shards: int, parity_shards: int, shard_size: int) -> np.ndarray:
    """encode_rs_u16_kernel, benchmark/rs/kernel.cu:67-102."""
    exp, _ = gf16_tables()
    d = data_padded[:data_shards * shard_size].reshape(data_shards, shard_size)
    shards = np.zeros((data_shards + parity_shards, shard_size), dtype=np.uint16)
    shards[:data_shards] = d
    for p in range(parity_shards):
        acc = np.zeros(shard_size, dtype=np.uint16)
        base = p + 1
        for k in range(data_shards):
            coef = exp[(base * k) % GF16_ORDER]
            acc ^= gf16_mul(d[k], coef)
        shards[data_shards + p] = acc
    return shards


def rs16_invert(missing_data, parity_used):
    """The per-block matrix build and Gauss-Jordan of
    reconstruct_rs_u16_kernel_inplace, benchmark/rs/kernel.cu:135-185."""
    exp, _ = gf16_tables()
    m = len(missing_data)
    V = [[int(exp[((parity_used[r] + 1) * missing_data[c]) % GF16_ORDER]) for c in range(m)] for r in range(m)]
    inv = [[1 if r == c else 0 for c in range(m)] for r in range(m)]
    for i in range(m):
        pr = i
        while pr < m and V[pr][i] == 0:
            pr += 1
        if pr == m:
            continue
        if pr != i:
            V[i], V[pr] = V[pr], V[i]
            inv[i], inv[pr] = inv[pr], inv[i]
        piv = V[i][i]
        if piv == 0:
            continue
        ip = gf16_div(1, piv)
        V[i] = [int(gf16_mul(x, ip)) for x in V[i]]
        inv[i] = [int(gf16_mul(x, ip)) for x in inv[i]]
        for r in range(m):
            if r == i:
                continue
            f = V[r][i]
            if f:
                V[r] = [V[r][c] ^ int(gf16_mul(f, V[i][c])) for c in range(m)]
                inv[r] = [inv[r][c] ^ int(gf16_mul(f, inv[i][c])) for c in range(m)]
    return inv


def rs16_reconstruct(shards: np.ndarray, data_shards: int, missing_data: list, parity_used: list) -> np.ndarray:
    """reconstruct_rs_u16_kernel_inplace, benchmark/rs/kernel.cu:105-222 (in place)."""
    m = len(missing_data)
    if m == 0:
        return shards
    exp, _ = gf16_tables()
    inv = rs16_invert(missing_data, parity_used)
    b = []
    for r in range(m):
        pr = parity_used[r]
        acc = shards[data_shards + pr].copy()
        base = pr + 1
        for k in range(data_shards):
            if k in missing_data:
                continue
            acc ^= gf16_mul(shards[k], exp[(base * k) % GF16_ORDER])
        b.append(acc)
    sols = []
    for c in range(m):
        s = np.zeros(shards.shape[1], dtype=np.uint16)
        for r in range(m):
            s ^= gf16_mul(np.uint16(inv[c][r]), b[r])
        sols.append(s)
    for c in range(m):
        shards[missing_data[c]] = sols[c]
    return shards


def rs16_forward_encode_kv(keys: np.ndarray, values: np.ndarray, num_data_shards: int, num_parity_shards: int):
    """forward_encode_kv, benchmark/rs/main.py:63-137 (byte work). Returns (shards, meta)."""
    B, H, T, D = keys.shape
    kv = np.concatenate([keys.reshape(-1), values.reshape(-1)]).astype(np.uint16)
    total = kv.size
    shard_sz, pad = shard_size_and_pad(total, num_data_shards)
    data_padded = np.zeros(num_data_shards * shard_sz, dtype=np.uint16)
    data_padded[:total] = kv
    shards = rs16_encode(data_padded, num_data_shards, num_parity_shards, shard_sz)
    meta = {"B": B, "H": H, "T": T, "D": D, "N_k": keys.size, "N_v": values.size, "total": total, "pad": pad,
            "shard_sz": shard_sz, "num_data": num_data_shards, "num_parity": num_parity_shards}
    return shards, meta


def rs16_backwards_decode_kv(shards: np.ndarray, meta: dict, missing_shards: list):
    """backwards_decode_kv, benchmark/rs/main.py:140-206 (in place on shards)."""
    nd, npar = meta["num_data"], meta["num_parity"]
    missing_data = sorted(i for i in missing_shards if i < nd)
    missing_par = sorted(i - nd for i in missing_shards if nd <= i < nd + npar)
    avail = [p for p in range(npar) if p not in missing_par]
    if len(missing_data) > len(avail):
        raise RuntimeError("Not enough parity shards to reconstruct the missing data shards.")
    if missing_data:
        if len(missing_data) > 16:
            raise RuntimeError("Reconstruction supports at most 16 missing data shards at once.")
        rs16_reconstruct(shards, nd, missing_data, avail[:len(missing_data)])
    data = shards[:nd].reshape(-1)[:meta["total"]]
    shp = (meta["B"], meta["H"], meta["T"], meta["D"])
    return data[:meta["N_k"]].reshape(shp), data[meta["N_k"]:meta["N_k"] + meta["N_v"]].reshape(shp)
