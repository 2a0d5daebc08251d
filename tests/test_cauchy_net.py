"""The bit-sliced RS(k, m) encoders' XOR networks (``csrc/cauchy_net.cuh``,
written by ``csrc/gen_cauchy_net.py``) replayed on the CPU: the committed
header is the generator's output, the pair elimination keeps every plane sum,
and bytes -> bit planes -> network -> bytes equals the oracle's RS(k, m)
encode over GF(2^8)/0x11d for every shape the library builds."""
from __future__ import annotations

import importlib.util
import os

import numpy as np
import pytest

from conftest import ROOT
from oracle import codes

_spec = importlib.util.spec_from_file_location(
    "gen_cauchy_net", os.path.join(ROOT, "26mlsys-ae-ghostserve_b200", "csrc", "gen_cauchy_net.py"))
gen = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(gen)

M32 = 0xFFFFFFFF


def test_header_is_generated():
    with open(gen.OUT) as f:
        assert f.read() == gen.render()


def transpose8(w):
    """Bit t of byte lane l of word s <-> bit s of byte lane l of word t."""
    w = list(w)
    for s, m, pairs in ((4, 0x0F0F0F0F, [(t, t + 4) for t in range(4)]),
                        (2, 0x33333333, [(0, 2), (1, 3), (4, 6), (5, 7)]),
                        (1, 0x55555555, [(t, t + 1) for t in range(0, 8, 2)])):
        for a, b in pairs:
            x = ((w[a] >> s) ^ w[b]) & m
            w[b] ^= x
            w[a] = (w[a] ^ (x << s)) & M32
    return w


def run_network(k, m, planes):
    temps, sums = gen.eliminate(k, m)
    var = [planes[v // 8][v % 8] for v in range(8 * k)]
    for a, b in temps:
        var.append(var[a] ^ var[b])
    out = [[0] * 8 for _ in range(m)]
    for q, s in enumerate(sums):
        acc = 0
        for v in s:
            acc ^= var[v]
        out[q // 8][q % 8] = acc
    return out


@pytest.mark.parametrize("k,m", gen.SHAPES)
def test_elimination_keeps_plane_sums(k, m):
    rng = np.random.default_rng(k * 10 + m)
    planes = [[int(x) for x in rng.integers(0, 1 << 32, 8, dtype=np.uint64)] for _ in range(k)]
    got = run_network(k, m, planes)
    for q, s in enumerate(gen.plane_sums(k, m)):
        acc = 0
        for v in s:
            acc ^= planes[v // 8][v % 8]
        assert got[q // 8][q % 8] == acc


@pytest.mark.parametrize("k,m", gen.SHAPES)
def test_bytes_through_planes_match_oracle(k, m):
    rng = np.random.default_rng(100 + k * 10 + m)
    nbytes = 32 * 12
    data = [rng.integers(0, 256, nbytes, dtype=np.uint8) for _ in range(k)]
    out = [np.zeros(nbytes, np.uint8) for _ in range(m)]
    for g in range(0, nbytes, 32):
        planes = [transpose8(d[g:g + 32].view(np.uint32).tolist()) for d in data]
        for j, o in enumerate(run_network(k, m, planes)):
            out[j][g:g + 32] = np.array(transpose8(o), np.uint32).view(np.uint8)
    for a, b in zip(out, codes.rs8_encode(data, m)):
        assert np.array_equal(a, b)


def test_generator_matches_oracle_coefficients():
    for k, m in gen.SHAPES:
        g = codes.rs8_generator(k, m)[k:]
        for j in range(m):
            for i in range(k):
                assert int(g[j][i]) == gen.gf_inv((k + j) ^ i)
