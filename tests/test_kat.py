"""Known answers for the engine's codes that do not come from ``oracle/codes.py``.

The reference has no code for textbook RDP (config 1) or RS(k,m) over GF(2^8)
(config 2). These tests pin both three ways: hand-derived cells, a second
restatement of the published algorithms (``tests/golden/kat.py``: bitwise field
arithmetic, brute-force inverses, a diagonal walk), and that restatement's
SHA-256 digests committed in ``tests/golden/kat_codes.json`` (which the GPU
tests and ``bench.py``'s default check compare the CUDA output against).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

from conftest import ROOT
from oracle import codes

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import kat  # noqa: E402


def fixture():
    with open(kat.KAT_FILE) as f:
        return json.load(f)


# ----------------------------------------------------------------- GF(2^8) ---
def test_field_facts():
    # x^8 = x^4 + x^3 + x^2 + 1 (0x1d) in GF(2^8)/0x11d
    x8 = 1
    for _ in range(8):
        x8 = kat.gf_mul(x8, 2)
    assert x8 == 0x1D
    # 2 generates the multiplicative group (order 255)
    seen, v = set(), 1
    for _ in range(255):
        seen.add(v)
        v = kat.gf_mul(v, 2)
    assert v == 1 and len(seen) == 255
    # 1/2 = 0x8e: 2 * 0x8e = 0x11c, reduced by 0x11d
    assert kat.gf_inv(2) == 0x8E and kat.gf_inv(3) == 0xF4
    rng = np.random.default_rng(5)
    for a, b, c in rng.integers(0, 256, (200, 3)):
        a, b, c = int(a), int(b), int(c)
        assert kat.gf_mul(a, b) == kat.gf_mul(b, a)
        assert kat.gf_mul(a, b ^ c) == kat.gf_mul(a, b) ^ kat.gf_mul(a, c)
        assert kat.gf_mul(a, b) == codes.gf8_mul_bitwise(a, b) == int(codes.gf8_mul(a, b))


def test_cauchy_6_2_matrix():
    # C[j][i] = 1 / ((6 + j) XOR i): row 0 is 1/6, 1/7, 1/4, 1/5, 1/2, 1/3
    want = [[122, 186, 71, 167, 142, 244], [186, 122, 167, 71, 244, 142]]
    assert kat.cauchy(6, 2) == want
    assert fixture()["cauchy_6_2"] == want
    assert codes.rs8_generator(6, 2)[6:].tolist() == want
    for row, x in zip(want, (6, 7)):
        for i, c in enumerate(row):
            assert kat.gf_mul(c, x ^ i) == 1


def test_rs8_multi_symbol_by_hand():
    # parity0 = 0x7a*d0 + 0xba*d1 + ... for two symbols, products by hand-checked rows
    d = [np.array([1, 0x80], np.uint8), np.array([2, 0], np.uint8), np.array([0, 0], np.uint8),
         np.array([0, 0], np.uint8), np.array([0, 0], np.uint8), np.array([1, 1], np.uint8)]
    p0, p1 = kat.rs8_encode(d, 2)
    # symbol 0: 0x7a*1 + 0xba*2 + 0xf4*1 ; 0xba*2 = 0x174 -> 0x174 ^ 0x11d = 0x69
    assert p0[0] == 0x7A ^ 0x69 ^ 0xF4
    # symbol 1: 0x7a*0x80 + 0xf4*1
    assert p0[1] == kat.gf_mul(0x7A, 0x80) ^ 0xF4
    assert p1[0] == 0xBA ^ kat.gf_mul(0x7A, 2) ^ 0x8E
    got = codes.rs8_encode(d, 2)
    assert got[0].tolist() == p0.tolist() and got[1].tolist() == p1.tolist()


# --------------------------------------------------------------------- RDP ---
def test_rdp_p7_cells_by_hand():
    # p=7, unit=1 byte, one stripe of 6 rows, six data disks.
    # D2[3] = 0xa5: P[3] = 0xa5; cell (3,2) is on diagonal 5, P's cell (3,6) on diagonal 2.
    # D1[5] = 0x3c: P[5] = 0x3c; cell (5,1) is on diagonal 6 (not stored), P's cell (5,6) on diagonal 4.
    data = [np.zeros(6, np.uint8) for _ in range(6)]
    data[2][3] = 0xA5
    data[1][5] = 0x3C
    P, Q = kat.rdp_encode(data, 7, 1)
    assert P.tolist() == [0, 0, 0, 0xA5, 0, 0x3C]
    assert Q.tolist() == [0, 0, 0xA5, 0, 0x3C, 0xA5]
    P2, Q2 = codes.rdp_encode(data, 7, 1)
    assert P2.tolist() == P.tolist() and Q2.tolist() == Q.tolist()


def test_rdp_p3_tail_stripe_by_hand():
    # p=3, k=2, unit=1: 3 bytes per shard -> 2 stripes, the second padded with a zero row
    a = np.array([1, 2, 3], np.uint8)
    b = np.array([4, 8, 12], np.uint8)
    P, Q = kat.rdp_encode([a, b], 3, 1)
    assert P.tolist() == [5, 10, 15, 0]
    # stripe 0: Q[0] = a0 ^ P1 (b's diagonal-0 cell is row 2: missing), Q[1] = a1 ^ b0
    # stripe 1: rows (3, 0): Q[0] = 3 ^ 0 = 3, Q[1] = 0 ^ 12 = 12
    assert Q.tolist() == [1 ^ 10, 2 ^ 4, 3, 12]


# ---------------------------------------------------- second restatement ---
SMALL = [c for c in kat.CASES if not c[0].startswith("config")]


@pytest.mark.parametrize("case", SMALL, ids=[c[0] for c in SMALL])
def test_small_cases_match_oracle_and_fixture(case):
    name, scheme, k, m, p, unit, kind, nbytes, seed = case
    data = kat.case_data(case)
    par = kat.case_parity(case, data)
    if scheme == "rdp":
        want = codes.rdp_encode(data, p, unit)
    elif scheme == "rs8":
        want = codes.rs8_encode(data, m)
    else:
        want = [codes.xor_encode(data)]
    assert len(want) == len(par) == m
    for a, b in zip(par, want):
        assert np.array_equal(a, b)
    rec = fixture()["cases"][name]
    assert [kat.sha(x) for x in par] == rec["parity_sha256"]


CONFIGS = [c for c in kat.CASES if c[0].startswith("config")]


@pytest.mark.parametrize("case", CONFIGS, ids=[c[0] for c in CONFIGS])
def test_config_cases_match_fixture_and_oracle(case):
    """Full benchmark sizes (32 MiB bf16 / 16 MiB fp8 shards): the second
    restatement reproduces the committed digests, and so does the oracle."""
    name, scheme, k, m, p, unit, kind, nbytes, seed = case
    data = kat.case_data(case)
    rec = fixture()["cases"][name]
    assert [kat.sha(x) for x in kat.case_parity(case, data)] == rec["parity_sha256"]
    if scheme == "rdp":
        want = codes.rdp_encode(data, p, unit)
    elif scheme == "rs8":
        want = codes.rs8_encode(data, m)
    else:
        want = [codes.xor_encode(data)]
    assert [kat.sha(x) for x in want] == rec["parity_sha256"]


def test_fixture_lists_every_case():
    f = fixture()["cases"]
    assert sorted(f) == sorted(c[0] for c in kat.CASES)
    for case in kat.CASES:
        rec = f[case[0]]
        assert (rec["scheme"], rec["k"], rec["m"], rec["p"], rec["unit"], rec["kind"], rec["shard_bytes"],
                rec["seed"]) == tuple(case[1:])


def test_bench_inputs_are_the_known_answer_cases():
    """bench.py restates the seeded generator (it imports nothing from tests/):
    the restatement must give the same bytes, and its workloads the sizes of
    the committed cases, so its parity check against the digests is valid."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    for kind in ("bf16", "u8"):
        for j in (0, 3):
            assert np.array_equal(bench.kat_shard(kind, 77, j, 4096), kat.shard_bytes(kind, 77, j, 4096))
    f = fixture()["cases"]
    for wl, case in bench.KAT_CASE.items():
        w, rec = bench.WORKLOADS[wl], f[case]
        assert (w["scheme"], w["k"], w["m"], w["p"], w["shard"]) == (rec["scheme"], rec["k"], rec["m"], rec["p"],
                                                                      rec["shard_bytes"])
        if w["scheme"] == "rdp":
            assert w["unit"] == rec["unit"]
        assert rec["kind"] == ("bf16" if w["kv"] == "bf16" else "u8")
