"""Pin the CPU oracle to the reference: the fixtures in tests/golden were produced
by the reference's own CUDA extensions (tests/golden/make_golden.py, run on a
B200 with the extensions built from the reference sources); the oracle must
reproduce every byte from the same inputs."""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import reference as R

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    path = os.path.join(GOLD, name)
    if not os.path.exists(path):
        pytest.fail(f"golden fixture {name} missing: run tests/golden/make_golden.py on a GPU box")
    z = np.load(path)
    cases = sorted({k.split("_", 1)[0] for k in z.files})
    return z, cases


def test_golden_xor():
    z, cases = load("ref_xor.npz")
    for c in cases:
        g = lambda k: z[f"{c}_{k}"]  # noqa: E731
        shape, k, miss = tuple(g("shape")), int(g("k")), int(g("miss"))
        kv = R.xor_pack_kv(g("keys"), g("values"))
        assert np.array_equal(kv, g("kv_bytes")), c
        s, _ = R.determine_shard_size(kv.size, k)
        dp = np.zeros(k * s, np.uint8)
        dp[:kv.size] = kv
        enc = R.xor_encode(dp, k, s)
        assert np.array_equal(enc, g("encoded")), c
        sh = enc.copy()
        sh[miss] = 0
        sh, rec = R.xor_reconstruct(sh, s, k, [miss])
        assert np.array_equal(sh, g("rebuilt")) and np.array_equal(rec, g("recovered")[0]), c
        total = int(np.prod(shape))
        assert np.array_equal(R.xor_unpack_kv(sh[:k].reshape(-1), total), g("unpacked")), c


def test_golden_rdpref():
    z, cases = load("ref_rdp.npz")
    for c in cases:
        g = lambda k: z[f"{c}_{k}"]  # noqa: E731
        shape = tuple(int(x) for x in g("shape"))
        nd, star, a, b = int(g("nd")), int(g("star")), int(g("a")), int(g("b"))
        enc, S, _ = R.rdpref_backup(g("keys"), g("values"), nd, star)
        assert np.array_equal(enc, g("encoded")), c
        sh = enc.copy()
        if b < 0:
            sh[a] = 0
        R.rdpref_recovery(sh, nd, S, star, a, b)
        assert np.array_equal(sh, g("recovered")), c
        B, H, T, D = shape
        assert np.array_equal(R.rdpref_load_full(sh, T, B * H * D, nd, S), g("out_tn")), c


def test_golden_rs16():
    z, cases = load("ref_rs16.npz")
    for c in cases:
        g = lambda k: z[f"{c}_{k}"]  # noqa: E731
        k, m, miss = int(g("k")), int(g("m")), [int(x) for x in g("miss")]
        enc, meta = R.rs16_forward_encode_kv(g("keys"), g("values"), k, m)
        assert np.array_equal(enc, g("encoded")), c
        sh = enc.copy()
        for i in miss:
            sh[i] = 0
        md = sorted(i for i in miss if i < k)
        mp = sorted(i - k for i in miss if i >= k)
        av = [q for q in range(m) if q not in mp][:len(md)]
        R.rs16_reconstruct(sh, k, md, av)
        assert np.array_equal(sh, g("recovered")), c


def test_golden_hook():
    z, cases = load("ref_hook.npz")
    for c in cases:
        g = lambda k: z[f"{c}_{k}"]  # noqa: E731
        world, elems, star = int(g("world")), int(g("elems")), int(g("star"))
        P, Q = R.hook_compute_parity(g("k_all"), g("v_all"), elems, star)
        rows = g("rows")
        assert np.array_equal(P, rows[world]) and np.array_equal(Q, rows[world + 1]), c
        for r in range(world):
            assert np.array_equal(rows[r, :elems], g("k_all")[r * elems:(r + 1) * elems])
