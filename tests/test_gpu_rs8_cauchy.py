"""The RS(k, m) encode over GF(2^8) for the shapes whose Cauchy generator is
built into the library as a bit-sliced XOR network (k + m <= 8, m <= 2), against
the CPU oracle: every shape, whole 32-byte groups, a last group of one 16-byte
vector, ranges that start on an odd vector, two-segment
shards split inside a group, and a parity re-encode through decode (erased
parity rows only: the same generator rows)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import pkg, rand_bytes
from oracle import codes

pytestmark = pytest.mark.gpu

SHAPES = [(k, m) for k in range(2, 8) for m in range(1, 3) if k + m <= 8]


@pytest.fixture(autouse=True)
def device_status_clean():
    yield
    assert pkg("codec").device_status(clear=True) == 0


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint8).reshape(-1)


@pytest.mark.parametrize("k,m", SHAPES, ids=[f"k{k}m{m}" for k, m in SHAPES])
@pytest.mark.parametrize("nbytes", [16, 48, 64 * 32, 16 * 129, (1 << 20) + 16])
def test_encode_matches_oracle(rng, k, m, nbytes):
    g = pkg()
    data = [rand_bytes(rng, nbytes) for _ in range(k)]
    got = [host(t) for t in g.encode(g.CodeSpec.rs8(k, m), [dev(d) for d in data])]
    for a, b in zip(got, codes.rs8_encode(data, m)):
        assert np.array_equal(a, b)


@pytest.mark.parametrize("k,m", [(6, 2), (3, 2), (7, 1)])
def test_ranges_and_segments(rng, k, m):
    g = pkg()
    spec = g.CodeSpec.rs8(k, m)
    nbytes = 16 * 301 + 16 * 257
    data = [rand_bytes(rng, nbytes) for _ in range(k)]
    want = codes.rs8_encode(data, m)
    # ranges cut at an odd 16-byte vector: the second starts mid-group
    par = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(m)]
    ddata = [dev(d) for d in data]
    cut = 16 * 37
    g.encode(spec, ddata, par, 0, cut)
    g.encode(spec, ddata, par, cut, nbytes)
    for a, b in zip(par, want):
        assert np.array_equal(host(a), b)
    # two segments per shard, split at 16 * 301 (inside a 32-byte group)
    pairs = [(dev(d[:16 * 301]), dev(d[16 * 301:])) for d in data]
    for a, b in zip(g.encode(spec, pairs), want):
        assert np.array_equal(host(a), b)


@pytest.mark.parametrize("k,m", [(6, 2), (4, 1)])
def test_parity_rebuild_through_decode(rng, k, m):
    g = pkg()
    spec = g.CodeSpec.rs8(k, m)
    nbytes = 16 * 515
    data = [rand_bytes(rng, nbytes) for _ in range(k)]
    want = codes.rs8_encode(data, m)
    er = list(range(k, k + m))
    sh = [dev(d) for d in data] + [None] * m
    out = g.decode(spec, sh, er, data_bytes=nbytes)
    for j in range(m):
        assert np.array_equal(host(out[k + j]), want[j])
