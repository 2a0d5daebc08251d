"""GPU parity of the engine codes (XOR, textbook RDP, RS8) against the CPU oracle.

Bit-exact on seeded inputs at small sizes for every erasure pattern; at the
benchmark sizes (32 MiB bf16 shards) through size-independent properties:
encode -> erase every pair -> decode returns the original bytes."""
from __future__ import annotations

import itertools

import numpy as np
import pytest
import torch

from conftest import pkg, rand_bytes
from oracle import codes

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def device_status_clean():
    """Every staged kernel's bounded waits completed (libgsec status word 0)."""
    yield
    assert pkg("codec").device_status(clear=True) == 0


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint8).reshape(-1)


def run_roundtrip(spec, data_np, erasure_sets, data_bytes):
    g = pkg()
    data = [dev(d) for d in data_np]
    par = g.encode(spec, data)
    full = [host(t) for t in data + par]
    for er in erasure_sets:
        shards = [None if i in er else (data + par)[i] for i in range(spec.n)]
        out = g.decode(spec, shards, er, data_bytes=data_bytes)
        for i in er:
            assert np.array_equal(host(out[i]), full[i]), (spec, er, i)
    return full


# ------------------------------------------------------------------- XOR -----
@pytest.mark.parametrize("k", [1, 2, 7, 8, 16])
@pytest.mark.parametrize("nbytes", [16, 4096, 16 * 1037])
def test_xor_matches_oracle(rng, k, nbytes):
    g = pkg()
    spec = g.CodeSpec.xor(k)
    data = [rand_bytes(rng, nbytes) for _ in range(k)]
    full = run_roundtrip(spec, data, [[e] for e in range(k + 1)], nbytes)
    assert np.array_equal(full[k], codes.xor_encode(data))


# ------------------------------------------------------------------- RDP -----
RDP_CASES = [(3, 2), (5, 4), (5, 3), (7, 6), (7, 4), (11, 8), (11, 10), (13, 12), (17, 16), (17, 9)]


@pytest.mark.parametrize("p,k", RDP_CASES)
@pytest.mark.parametrize("unit", [16, 4096])
def test_rdp_encode_matches_oracle(rng, p, k, unit):
    g = pkg()
    spec = g.CodeSpec.rdp(k, p, unit)
    data_bytes = 2 * (p - 1) * unit + 3 * unit + 32  # two stripes + a partial one
    data = [rand_bytes(rng, data_bytes) for _ in range(k)]
    P, Q = codes.rdp_encode(data, p, unit)
    par = g.encode(spec, [dev(d) for d in data])
    assert np.array_equal(host(par[0]), P)
    assert np.array_equal(host(par[1]), Q)


@pytest.mark.parametrize("p,k", RDP_CASES)
@pytest.mark.parametrize("unit", [64, 1024])  # per-thread kernel, TMA-staged kernel
def test_rdp_decodes_every_pattern(rng, p, k, unit):
    g = pkg()
    spec = g.CodeSpec.rdp(k, p, unit)
    data_bytes = 3 * (p - 1) * unit + 5 * 16
    data = [rand_bytes(rng, data_bytes) for _ in range(k)]
    pats = [list(e) for n in (1, 2) for e in itertools.combinations(range(k + 2), n)]
    run_roundtrip(spec, data, pats, data_bytes)


def test_rdp_decode_matches_oracle_peeling(rng):
    # CUDA mask decoder vs the oracle's independent peeling decoder.
    g = pkg()
    p, k, unit = 7, 6, 4096
    spec = g.CodeSpec.rdp(k, p, unit)
    data_bytes = 2 * 6 * unit + 4096
    data = [rand_bytes(rng, data_bytes) for _ in range(k)]
    P, Q = codes.rdp_encode(data, p, unit)
    full = data + [P, Q]
    ddata = [dev(d) for d in data]
    dpar = [dev(P), dev(Q)]
    for er in itertools.combinations(range(k + 2), 2):
        want = codes.rdp_decode([None if i in er else full[i] for i in range(k + 2)], k, p, unit, data_bytes)
        sh = [None if i in er else (ddata + dpar)[i] for i in range(k + 2)]
        out = g.decode(spec, sh, list(er), data_bytes=data_bytes)
        for i in er:
            assert np.array_equal(host(out[i]), want[i])


# ------------------------------------------------------------------- RS8 -----
@pytest.mark.parametrize("k,m", [(6, 2), (4, 4), (10, 3), (1, 1), (32, 4), (3, 2)])
def test_rs8_matches_oracle_every_pattern(rng, k, m):
    g = pkg()
    spec = g.CodeSpec.rs8(k, m)
    nbytes = 16 * 129
    data = [rand_bytes(rng, nbytes) for _ in range(k)]
    want = codes.rs8_encode(data, m)
    pats = [list(e) for n in range(1, m + 1) for e in itertools.combinations(range(k + m), n)]
    if len(pats) > 120:
        pats = pats[:: len(pats) // 120 + 1] + [list(range(k, k + m)), list(range(m))]
    full = run_roundtrip(spec, data, pats, nbytes)
    for j in range(m):
        assert np.array_equal(full[k + j], want[j])


# ---------------------------------------------------- segments and ranges ----
@pytest.mark.parametrize("scheme", ["xor", "rdp", "rdp4k", "rs8"])
def test_two_segment_shards_equal_concatenation(rng, scheme):
    g = pkg()
    k = 6
    spec = {"xor": g.CodeSpec.xor(k), "rdp": g.CodeSpec.rdp(k, 7, 256), "rs8": g.CodeSpec.rs8(k, 2),
            "rdp4k": g.CodeSpec.rdp(k, 7, 4096)}[scheme]
    # the split falls inside a 1 KiB staging segment (TMA kernels copy it in two parts)
    lo_b, hi_b = (16 * 301, 16 * 257) if scheme != "rdp4k" else (6 * 4096 + 16 * 301, 6 * 4096 + 16 * 257)
    lo = [rand_bytes(rng, lo_b) for _ in range(k)]
    hi = [rand_bytes(rng, hi_b) for _ in range(k)]
    cat = [dev(np.concatenate([a, b])) for a, b in zip(lo, hi)]
    pairs = [(dev(a), dev(b)) for a, b in zip(lo, hi)]
    want = [host(t) for t in g.encode(spec, cat)]
    got = [host(t) for t in g.encode(spec, pairs)]
    for a, b in zip(want, got):
        assert np.array_equal(a, b)
    # decode a data shard back into a split destination
    er = [1, k] if spec.m > 1 else [1]
    par = [dev(w) for w in want]
    dst = (torch.empty(lo_b, dtype=torch.uint8, device="cuda"), torch.empty(hi_b, dtype=torch.uint8, device="cuda"))
    sh = [p if i not in er else None for i, p in enumerate(pairs)] + list(par)
    sh[1] = dst
    if k in er:
        sh[k] = torch.empty_like(par[0])
    out = g.decode(spec, sh, er)
    assert np.array_equal(host(out[1][0]), lo[1]) and np.array_equal(host(out[1][1]), hi[1])


@pytest.mark.parametrize("scheme", ["xor", "rdp", "rs8"])
def test_range_slices_compose(rng, scheme):
    g = pkg()
    k = 4
    spec = {"xor": g.CodeSpec.xor(k), "rdp": g.CodeSpec.rdp(k, 5, 64), "rs8": g.CodeSpec.rs8(k, 3)}[scheme]
    nbytes = 4 * 256 * 7 + 64
    data = [dev(rand_bytes(rng, nbytes)) for _ in range(k)]
    full = [host(t) for t in g.encode(spec, data)]
    pb = spec.parity_bytes(nbytes)
    gran = spec.stripe_bytes()
    cut = (pb // gran // 2) * gran
    par = [torch.zeros(pb, dtype=torch.uint8, device="cuda") for _ in range(spec.m)]
    g.encode(spec, data, par, 0, cut)
    g.encode(spec, data, par, cut, pb)
    for a, b in zip(full, par):
        assert np.array_equal(a, host(b))


# -------------------------------------------------------- benchmark sizes ----
def kv_shards_bf16(seed: int, k: int):
    """k ranks' KV chunk: K and V [32 layers, 2048 tokens, 1 head, 128] bf16 N(0,1)."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    out = []
    for _ in range(k):
        kv = torch.randn(2, 32, 2048, 1, 128, generator=gen, device="cuda", dtype=torch.float32).to(torch.bfloat16)
        out.append(kv.view(torch.uint8).reshape(-1))
    return out


def test_config1_rdp_p7_full_size_all_pairs():
    g = pkg()
    spec = g.CodeSpec.rdp(6, 7, 4096)
    data = kv_shards_bf16(11, 6)
    assert data[0].numel() == 32 << 20
    par = g.encode(spec, data)
    assert par[0].numel() == 1366 * 6 * 4096
    full = data + par
    sums = [torch.sum(t.view(torch.int32).to(torch.int64)).item() for t in full]
    for er in itertools.combinations(range(8), 2):
        sh = [None if i in er else full[i] for i in range(8)]
        out = g.decode(spec, sh, list(er), data_bytes=32 << 20)
        for i in er:
            assert torch.equal(out[i], full[i]), er
            assert torch.sum(out[i].view(torch.int32).to(torch.int64)).item() == sums[i]


def test_config1_matches_oracle_on_a_slice():
    g = pkg()
    spec = g.CodeSpec.rdp(6, 7, 4096)
    data = kv_shards_bf16(12, 6)
    par = g.encode(spec, data)
    sb = 6 * 4096
    lo, hi = 500 * sb, 503 * sb
    want = codes.rdp_encode([host(d[lo:hi]) for d in data], 7, 4096)
    assert np.array_equal(host(par[0][lo:hi]), want[0])
    assert np.array_equal(host(par[1][lo:hi]), want[1])
    # the padded tail stripe
    tail = 1365 * sb
    want = codes.rdp_encode([host(d[tail:]) for d in data], 7, 4096)
    assert np.array_equal(host(par[0][tail:]), want[0])
    assert np.array_equal(host(par[1][tail:]), want[1])


def test_config2_rs8_fp8_full_size_all_pairs():
    g = pkg()
    spec = g.CodeSpec.rs8(6, 2)
    gen = torch.Generator(device="cuda").manual_seed(21)
    data = [torch.randint(0, 256, (16 << 20,), generator=gen, device="cuda", dtype=torch.uint8) for _ in range(6)]
    par = g.encode(spec, data)
    full = data + par
    for er in itertools.combinations(range(8), 2):
        out = g.decode(spec, [None if i in er else full[i] for i in range(8)], list(er), data_bytes=16 << 20)
        for i in er:
            assert torch.equal(out[i], full[i]), er
    lo = 4096 * 100
    want = codes.rs8_encode([host(d[lo:lo + 4096]) for d in data], 2)
    assert np.array_equal(host(par[0][lo:lo + 4096]), want[0])
    assert np.array_equal(host(par[1][lo:lo + 4096]), want[1])


def test_config0_xor_full_size():
    g = pkg()
    spec = g.CodeSpec.xor(7)
    data = kv_shards_bf16(3, 7)
    par = g.encode(spec, data)
    x = data[0].clone()
    for d in data[1:]:
        x ^= d
    assert torch.equal(x, par[0])
    gen = np.random.default_rng(5)
    e = int(gen.integers(0, 8))
    full = data + par
    out = g.decode(spec, [None if i == e else full[i] for i in range(8)], [e], data_bytes=32 << 20)
    assert torch.equal(out[e], full[e])


# ------------------------------------------------------- pool rows by slot ---
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("heads", [1, 2, 8])
def test_slots_gather_scatter_match_fancy_indexing(dtype, heads):
    codec = pkg("codec")
    pool = torch.randn(1000, 2, heads, 128, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(1000, device="cuda")[:333].to(dtype)
    slots[::7] = -1
    row = heads * 128 * 2
    for plane in (0, 1):
        out = torch.empty(333 * row + 64, dtype=torch.uint8, device="cuda")
        codec.slots_gather(pool, slots, out, plane=plane)
        want = pool[slots.long().clamp(min=0), plane].clone()
        want[slots.long() < 0] = 0
        assert torch.equal(out[:333 * row], want.reshape(-1).view(torch.uint8))
    # scatter puts rows back exactly where gather took them; -1 rows untouched
    src = torch.randint(0, 256, (333 * row,), dtype=torch.uint8, device="cuda")
    before = pool.clone()
    codec.slots_scatter(pool, slots, src, plane=1)
    s = slots.long()
    expect = before.clone()
    expect[s[s >= 0], 1] = src.view(torch.bfloat16).view(333, heads, 128)[s >= 0]
    assert torch.equal(pool.view(torch.int16), expect.view(torch.int16))  # random bytes include NaNs


def test_slots_gather_flags_a_slot_past_the_pool():
    codec = pkg("codec")
    pool = torch.zeros(64, 2, 1, 128, device="cuda", dtype=torch.bfloat16)
    slots = torch.tensor([3, 64, 5], device="cuda")
    out = torch.full((3 * 256,), 7, dtype=torch.uint8, device="cuda")
    codec.slots_gather(pool, slots, out)
    assert codec.device_status(clear=True) == 1 << 16
    assert int(out[256:512].sum()) == 0  # the bad row is zeroed, not read


def test_slots_gather_rejects_bad_arguments():
    codec = pkg("codec")
    pool = torch.zeros(64, 2, 1, 128, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        codec.slots_gather(pool, torch.tensor([1, 2], device="cuda", dtype=torch.int16), out)
    with pytest.raises(ValueError):
        codec.slots_gather(pool, torch.arange(40, device="cuda"), out[:100])
    with pytest.raises(ValueError):
        wide = torch.zeros(64, 2, 2, 128, device="cuda", dtype=torch.bfloat16)
        codec.slots_gather(wide[:, :, :, :64], torch.arange(4, device="cuda"), out)  # rows not contiguous
    with pytest.raises(ValueError):
        codec.slots_gather(pool, torch.arange(4, device="cuda"), out[1:])  # misaligned buffer


# ------------------------------------------------------------ bulk gather ---
@pytest.mark.parametrize("sizes", [[16], [0, 48, 16384], [16384 * 3 + 32, 7 * 16, 65536, 0, 16400], [1 << 20] * 5])
def test_copy_gather_concatenates(sizes):
    L = pkg("_lib")
    g = torch.Generator(device="cuda").manual_seed(len(sizes))
    srcs = [torch.randint(0, 256, (max(n, 16),), generator=g, device="cuda", dtype=torch.uint8) for n in sizes]
    dst = torch.full((sum(sizes) + 64,), 7, dtype=torch.uint8, device="cuda")
    ptrs = L.ptr_array([t.data_ptr() for t in srcs])
    nb = (L.C.c_int64 * len(sizes))(*sizes)
    L.call("gsec_copy_gather", ptrs, nb, len(sizes), L.C.c_void_p(dst.data_ptr()),
           L.C.c_void_p(torch.cuda.current_stream().cuda_stream))
    want = torch.cat([t[:n] for t, n in zip(srcs, sizes)])
    assert torch.equal(dst[:sum(sizes)], want)
    assert int((dst[sum(sizes):] == 7).sum()) == 64  # nothing past the end
