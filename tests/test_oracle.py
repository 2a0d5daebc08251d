"""CPU checks of the oracle itself: field tables, hand-computed known-answer
vectors, and decode properties (every erasure pattern the code promises)."""
from __future__ import annotations

import itertools

import numpy as np
import pytest

from oracle import codes, reference as R
from conftest import fp16_bits, rand_bytes


# ----------------------------------------------------------------- fields ----
def test_gf16_reference_poly_is_primitive():
    exp, log = R.init_gf_tables()
    head = exp[:R.GF16_ORDER].astype(np.int64)
    assert np.unique(head).size == R.GF16_ORDER and head.min() == 1  # x generates all non-zero elements
    assert np.array_equal(exp[R.GF16_ORDER:], exp[:R.GF16_ORDER])
    assert np.all(log[exp[:R.GF16_ORDER]] == np.arange(R.GF16_ORDER))


def test_gf16_table_multiply_matches_polynomial_multiply(rng):
    def polymul(a, b):
        r = 0
        for _ in range(16):
            if b & 1:
                r ^= a
            b >>= 1
            a <<= 1
            if a & 0x10000:
                a ^= 0x1100B
        return r

    a = rng.integers(0, 1 << 16, 300)
    b = rng.integers(0, 1 << 16, 300)
    got = R.gf16_mul(a, b)
    assert all(int(g) == polymul(int(x), int(y)) for g, x, y in zip(got, a, b))


def test_gf8_tables_match_bitwise_multiply():
    a, b = np.meshgrid(np.arange(256), np.arange(256))
    t = codes.gf8_mul(a.ravel(), b.ravel())
    for x, y, v in zip(a.ravel()[::97], b.ravel()[::97], t[::97]):
        assert int(v) == codes.gf8_mul_bitwise(int(x), int(y))
    assert np.unique(codes.GF8_EXP[:255]).size == 255  # 0x11d is primitive
    for x in range(1, 256):
        assert codes.gf8_mul_bitwise(x, codes.gf8_inv(x)) == 1


# ------------------------------------------------------- known answers -------
def test_kat_rdpref_parity_with_star():
    # nd=2, S=3, star_base=0: P = D0^D1; Q[d] = D0[d] ^ D1[(d-1)%3] minus the star
    # cells (row0 col0 -> skipped at d=0, row1 col1 -> skipped at d=2).
    sh = np.zeros((4, 3), dtype=np.uint16)
    sh[0] = [1, 2, 4]
    sh[1] = [8, 16, 32]
    R.rdpref_parity(sh, 2, 3, 0)
    assert sh[2].tolist() == [9, 18, 36]
    assert sh[3].tolist() == [32, 10, 4]


def test_kat_rdpref_negative_star_never_skips():
    sh = np.zeros((4, 3), dtype=np.uint16)
    sh[0] = [1, 2, 4]
    sh[1] = [8, 16, 32]
    R.rdpref_parity(sh, 2, 3, -5)  # (-5 + r) % 3 is negative in C for r=0,1
    assert sh[3].tolist() == [1 ^ 32, 2 ^ 8, 4 ^ 16]


def test_kat_rs16_reference_coefficients():
    # P_p = sum_k alpha^((p+1)k) D_k with alpha = x = 2: k=2, D=[1],[1]
    sh = R.rs16_encode(np.array([1, 1], dtype=np.uint16), 2, 2, 1)
    assert sh[2, 0] == 1 ^ 2  # alpha^0 + alpha^1
    assert sh[3, 0] == 1 ^ 4  # alpha^0 + alpha^2


def test_kat_rdp_p3_unit1():
    # p=3, k=2, unit=1 byte: a=[1,2], b=[4,8] (rows 0,1)
    # P = [a0^b0, a1^b1]; Q[0] = a0 ^ b1... cells on diag 0: (0,0) and (1,2)=P1
    P, Q = codes.rdp_encode([np.array([1, 2], np.uint8), np.array([4, 8], np.uint8)], 3, 1)
    assert P.tolist() == [5, 10]
    assert Q.tolist() == [1 ^ 10, 2 ^ 4]


def test_kat_rs8_cauchy():
    # k=2, m=1: C = [1/(2^0), 1/(2^1)] = [1/2, 1/3] = [0x8e, 0xf4] in GF(2^8)/0x11d
    assert codes.gf8_inv(2) == 0x8E and codes.gf8_inv(3) == 0xF4
    (par,) = codes.rs8_encode([np.array([1], np.uint8), np.array([1], np.uint8)], 1)
    assert par.tolist() == [0x8E ^ 0xF4]


# -------------------------------------------------------- XOR (reference) ----
@pytest.mark.parametrize("k", [1, 2, 3, 7, 8])
def test_xor_reference_roundtrip_every_shard(rng, k):
    shape = (1, 2, 5, 8)
    keys, vals = fp16_bits(rng, shape), fp16_bits(rng, shape)
    shards, s, pad = R.xor_forward_encode_kv(keys, vals, k)
    assert s * k - pad == 4 * keys.size
    for miss in range(k + 1):
        kk, vv, rebuilt = R.xor_backwards_decode_kv(shards, shape, k, [miss])
        assert np.array_equal(kk, keys) and np.array_equal(vv, vals)
        assert np.array_equal(rebuilt, shards)


# ------------------------------------------------------- RDP (reference) -----
@pytest.mark.parametrize("nd,S,star", [(2, 3, 0), (3, 17, 1), (4, 300, 7), (8, 515, 0), (5, 256, 3), (6, 64, -2)])
def test_rdpref_recovery_sequence_reduces_to_closed_form(rng, nd, S, star):
    base = np.zeros((nd + 2, S), dtype=np.uint16)
    base[:nd] = rng.integers(0, 1 << 16, size=(nd, S), dtype=np.uint16)
    R.rdpref_parity(base, nd, S, star)
    pairs = [(0, 1), (1, 0), (0, nd - 1), (nd - 1, -1), (-1, 0), (1, 1), (nd, 0), (-1, -1)]
    for a, b in pairs:
        for erase in (False, True):
            sh = base.copy()
            if erase:  # zero the rows the caller reports missing
                for m in (a, b):
                    if 0 <= m < nd:
                        sh[m] = 0
            lit = R.rdpref_recovery(sh.copy(), nd, S, star, a, b)
            closed = R.rdpref_recovery_outcome(sh.copy(), nd, a, b)
            assert np.array_equal(lit, closed), (a, b, erase)


def test_rdpref_single_erasure_recovers(rng):
    keys, vals = fp16_bits(rng, (1, 2, 7, 8)), fp16_bits(rng, (1, 2, 7, 8))
    sh, S, _ = R.rdpref_backup(keys, vals, 5, 0)
    for a in range(5):
        e = sh.copy()
        e[a] = 0
        R.rdpref_recovery(e, 5, S, 0, a, -1)
        assert np.array_equal(e, sh)
        out = R.rdpref_load_full(e, 7, 16, 5, S)
        assert np.array_equal(R.from_tn(out[:7 * 16].reshape(7, 16), keys.shape), keys)


def _gf2_rank(m: np.ndarray) -> int:
    m = m.copy() % 2
    rank = 0
    for c in range(m.shape[1]):
        piv = next((r for r in range(rank, m.shape[0]) if m[r, c]), None)
        if piv is None:
            continue
        m[[rank, piv]] = m[[piv, rank]]
        for r in range(m.shape[0]):
            if r != rank and m[r, c]:
                m[r] ^= m[rank]
        rank += 1
    return rank


@pytest.mark.parametrize("nd,S", [(4, 7), (6, 8), (8, 16), (8, 17)])
def test_rdpref_pairs_are_not_recoverable(nd, S):
    """GF(2) rank of the map (erased rows a, b) -> (P, Q) of the reference code is
    below 2S for every pair: its P/Q cannot rebuild two data rows."""
    for a, b in itertools.combinations(range(nd), 2):
        cols = []
        for row in (a, b):
            for c in range(S):
                t = np.zeros((nd + 2, S), dtype=np.uint16)
                t[row, c] = 1
                R.rdpref_parity(t, nd, S, 0)
                cols.append(np.concatenate([t[nd], t[nd + 1]]).astype(np.int64))
        assert _gf2_rank(np.stack(cols, axis=1)) < 2 * S, (a, b)


def test_hook_parity_matches_benchmark_parity(rng):
    world, elems = 4, 24
    k_all = fp16_bits(rng, world * elems)
    v_all = fp16_bits(rng, world * elems)
    P, Q = R.hook_compute_parity(k_all, v_all, elems, star_base=2)
    rows = np.zeros((world + 2, 2 * elems), dtype=np.uint16)
    for r in range(world):
        rows[r, :elems] = k_all[r * elems:(r + 1) * elems]
        rows[r, elems:] = v_all[r * elems:(r + 1) * elems]
    R.rdpref_parity(rows, world, 2 * elems, 2)
    assert np.array_equal(P, rows[world]) and np.array_equal(Q, rows[world + 1])


# ------------------------------------------------------- RS16 (reference) ----
def test_rs16_reference_roundtrip_all_data_pairs(rng):
    keys, vals = fp16_bits(rng, (1, 1, 6, 8)), fp16_bits(rng, (1, 1, 6, 8))
    shards, meta = R.rs16_forward_encode_kv(keys, vals, 4, 2)
    for miss in itertools.combinations(range(6), 2):
        e = shards.copy()
        for m in miss:
            e[m] = 0
        kk, vv = R.rs16_backwards_decode_kv(e, meta, list(miss))
        assert np.array_equal(kk, keys) and np.array_equal(vv, vals), miss


def test_rs16_reference_not_enough_parity():
    keys = np.zeros((1, 1, 2, 4), np.uint16)
    shards, meta = R.rs16_forward_encode_kv(keys, keys, 3, 1)
    with pytest.raises(RuntimeError):
        R.rs16_backwards_decode_kv(shards, meta, [0, 1])


# ------------------------------------------------------- textbook RDP --------
@pytest.mark.parametrize("p,k", [(3, 2), (5, 4), (5, 2), (7, 6), (7, 3), (11, 8), (13, 12)])
def test_rdp_every_double_erasure_decodes(rng, p, k):
    unit = 16
    data_bytes = (p - 1) * unit * 2 + 48  # two full stripes and a partial one
    data = [rand_bytes(rng, data_bytes) for _ in range(k)]
    P, Q = codes.rdp_encode(data, p, unit)
    full = data + [P, Q]
    for ne in (1, 2):
        for er in itertools.combinations(range(k + 2), ne):
            sh = [None if i in er else full[i] for i in range(k + 2)]
            out = codes.rdp_decode(sh, k, p, unit, data_bytes)
            for i in er:
                assert np.array_equal(out[i], full[i]), (p, k, er)


def test_rdp_is_linear(rng):
    p, unit, k = 7, 32, 6
    a = [rand_bytes(rng, 6 * 32) for _ in range(k)]
    b = [rand_bytes(rng, 6 * 32) for _ in range(k)]
    pa, qa = codes.rdp_encode(a, p, unit)
    pb, qb = codes.rdp_encode(b, p, unit)
    pc, qc = codes.rdp_encode([x ^ y for x, y in zip(a, b)], p, unit)
    assert np.array_equal(pc, pa ^ pb) and np.array_equal(qc, qa ^ qb)


# ---------------------------------------------------------------- RS8 --------
@pytest.mark.parametrize("k,m", [(6, 2), (4, 4), (2, 2), (10, 3)])
def test_rs8_every_erasure_pattern_decodes(rng, k, m):
    g = codes.rs8_generator(k, m)
    for rows in itertools.combinations(range(k + m), k):  # MDS: any k rows invertible
        codes.gf8_invert(g[list(rows)])
    data = [rand_bytes(rng, 40) for _ in range(k)]
    full = data + codes.rs8_encode(data, m)
    for ne in range(1, m + 1):
        for er in itertools.combinations(range(k + m), ne):
            out = codes.rs8_decode([None if i in er else full[i] for i in range(k + m)], k, m)
            for i in er:
                assert np.array_equal(out[i], full[i])


def test_xor_generic_roundtrip(rng):
    data = [rand_bytes(rng, 64) for _ in range(5)]
    full = data + [codes.xor_encode(data)]
    for e in range(6):
        out = codes.xor_decode([None if i == e else full[i] for i in range(6)])
        assert np.array_equal(out[e], full[e])
