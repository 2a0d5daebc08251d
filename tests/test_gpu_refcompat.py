"""GPU parity of the reference-compatible drop-ins against the oracle's
restatement of the reference, and (when oracle/_ref is built) against the
reference's own CUDA extensions run on the same inputs."""
from __future__ import annotations

import itertools

import numpy as np
import pytest
import torch

from conftest import fp16_bits, pkg
from oracle import reference as R

pytestmark = pytest.mark.gpu

SHAPES = [(1, 8, 256, 128), (1, 2, 5, 8), (2, 3, 7, 16), (1, 1, 1, 8), (1, 2, 33, 24)]


def kv16(rng, shape, dtype=torch.float16):
    k, v = fp16_bits(rng, shape), fp16_bits(rng, shape)
    tk = torch.from_numpy(k).cuda().view(dtype)
    tv = torch.from_numpy(v).cuda().view(dtype)
    return k, v, tk, tv


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint16).cpu().numpy() if t.dtype != torch.uint8 else t.cpu().numpy()


def ref_mod(name):
    build_ref = pytest.importorskip("oracle.build_ref")
    if not build_ref.built(name):
        pytest.skip(f"reference extension {name} not built")
    return build_ref.load_ref(name)


# ------------------------------------------------------------------- XOR -----
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("k", [1, 3, 7, 8])
def test_xor_dropin_matches_reference_math(rng, shape, k):
    x = pkg("benchmark.xor.main")
    kn, vn, kt, vt = kv16(rng, shape)
    pkg_ = x.forward_encode_kv(kt, vt, k, 1)
    want, s, pad = R.xor_forward_encode_kv(kn, vn, k)
    assert pkg_["shard_size"] == s and pkg_["pad"] == pad
    assert np.array_equal(pkg_["shards_KV"].cpu().numpy(), want)
    for miss in range(k + 1):
        ko, vo, st = x.backwards_decode_kv(pkg_, [miss])
        assert np.array_equal(u16(ko), kn) and np.array_equal(u16(vo), vn)
        assert np.array_equal(pkg_["shards_KV"].cpu().numpy(), want)
        assert st["reconstruct_io"] == 0 and "unpack_io" in st


def test_xor_dropin_errors(rng):
    x = pkg("benchmark.xor.main")
    _, _, kt, vt = kv16(rng, (1, 1, 4, 8))
    p = x.forward_encode_kv(kt, vt, 4, 1)
    with pytest.raises(ValueError):
        x.backwards_decode_kv(p, [0, 1])
    with pytest.raises(ValueError):
        x.backwards_decode_kv(p, [5])


def test_xor_dropin_bf16_raw_bytes(rng):
    x = pkg("benchmark.xor.main")
    kn, vn, kt, vt = kv16(rng, (1, 2, 9, 8), torch.bfloat16)
    p = x.forward_encode_kv(kt, vt, 5, 1)
    want, _, _ = R.xor_forward_encode_kv(kn, vn, 5)
    assert np.array_equal(p["shards_KV"].cpu().numpy(), want)
    ko, vo, _ = x.backwards_decode_kv(p, [2])
    assert ko.dtype == torch.bfloat16 and np.array_equal(u16(ko), kn)


def test_xor_ext_level_names(rng):
    e = pkg("ext")
    kn, vn, kt, vt = kv16(rng, (1, 2, 6, 8))
    T, n = 6, 16
    kvb = torch.empty(4 * T * n, dtype=torch.uint8, device="cuda")
    e.xor_kernel.pack_kv(kt, vt, kvb, n, T)
    assert np.array_equal(kvb.cpu().numpy(), R.xor_pack_kv(kn, vn))
    k, s = 3, (4 * T * n + 2) // 3
    dp = torch.zeros(k * s, dtype=torch.uint8, device="cuda")
    dp[:kvb.numel()] = kvb
    sh = torch.zeros((k + 1, s), dtype=torch.uint8, device="cuda")
    e.xor_kernel.encode_xor(dp, sh, k, s)
    want = R.xor_encode(dp.cpu().numpy(), k, s)
    assert np.array_equal(sh.cpu().numpy(), want)
    sh[1].zero_()
    rec = torch.empty((1, s), dtype=torch.uint8, device="cuda")
    e.xor_kernel.reconstruct_xor(sh, sh, rec, s, k, torch.tensor([1], dtype=torch.int32, device="cuda"))
    assert np.array_equal(sh.cpu().numpy(), want) and np.array_equal(rec.cpu().numpy()[0], want[1])
    out = torch.empty(2 * T * n, dtype=torch.float16, device="cuda")
    e.xor_kernel.unpack_kv(kvb, out, n, T)
    assert np.array_equal(u16(out), np.concatenate([kn.reshape(-1), vn.reshape(-1)]))


# ------------------------------------------------------------------- RDP -----
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("nd,star", [(8, 0), (6, 3), (3, 1), (2, -1), (5, 1000)])
def test_rdpref_backup_matches_reference_math(rng, shape, nd, star):
    r = pkg("benchmark.rdp.main")
    kn, vn, kt, vt = kv16(rng, shape)
    p = r.fused_backup_full_kv(kt, vt, nd, star_base=star)
    want, S, pad = R.rdpref_backup(kn, vn, nd, star)
    assert p["shard_size"] == S and p["pad_words"] == pad
    assert np.array_equal(p["shards_KV"].cpu().numpy(), want)


@pytest.mark.parametrize("shape", SHAPES[:3])
def test_rdpref_recovery_matches_reference_sequence(rng, shape):
    r = pkg("benchmark.rdp.main")
    nd = 6
    kn, vn, kt, vt = kv16(rng, shape)
    p = r.fused_backup_full_kv(kt, vt, nd, star_base=2)
    base = p["shards_KV"].clone()
    S = p["shard_size"]
    for a, b in [(0, 1), (3, -1), (-1, 5), (4, 2), (2, 2), (nd, 1), (-1, -1)]:
        for erase in (False, True):
            p["shards_KV"].copy_(base)
            if erase:
                for m in (a, b):
                    if 0 <= m < nd:
                        p["shards_KV"][m].zero_()
            before = p["shards_KV"].cpu().numpy()
            ko, vo, st = r.fused_recovery_full_kv(p, a, b)
            want = R.rdpref_recovery(before.copy(), nd, S, 2, a, b)
            assert np.array_equal(p["shards_KV"].cpu().numpy(), want), (a, b, erase)
            B, H, T, D = shape
            tn = R.rdpref_load_full(want, T, B * H * D, nd, S)
            assert np.array_equal(u16(ko), R.from_tn(tn[:T * B * H * D].reshape(T, -1), shape))
            assert np.array_equal(u16(vo), R.from_tn(tn[T * B * H * D:].reshape(T, -1), shape))
            if not erase or (a < 0 or a >= nd) and (b < 0 or b >= nd):
                assert np.array_equal(u16(ko), kn) and np.array_equal(u16(vo), vn)
            assert st["recover_ms"] >= 0


def test_rdpref_single_erasure_restores_kv(rng):
    r = pkg("benchmark.rdp.main")
    kn, vn, kt, vt = kv16(rng, (1, 8, 64, 128))
    p = r.fused_backup_full_kv(kt, vt, 8)
    for a in range(8):
        p2 = dict(p)
        p2["shards_KV"] = p["shards_KV"].clone()
        p2["shards_KV"][a].zero_()
        ko, vo, _ = r.fused_recovery_full_kv(p2, a)
        assert np.array_equal(u16(ko), kn) and np.array_equal(u16(vo), vn)


def test_rdp_ext_level_tn(rng):
    e = pkg("ext")
    kn, vn, kt, vt = kv16(rng, (1, 2, 9, 8))
    T, n, nd = 9, 16, 4
    S, _ = R.determine_shard_size_words(2 * T * n, nd)
    ktn = torch.from_numpy(R.to_tn(kn)).cuda().view(torch.float16)
    vtn = torch.from_numpy(R.to_tn(vn)).cuda().view(torch.float16)
    sh = torch.zeros((nd + 2, S), dtype=torch.uint16, device="cuda")
    e.rdp_kernel.fused_backup_full_kv(ktn, vtn, sh, nd, S, T, n, 1)
    want, _, _ = R.rdpref_backup(kn, vn, nd, 1)
    assert np.array_equal(sh.cpu().numpy(), want)
    out = torch.empty(2 * T * n, dtype=torch.float16, device="cuda")
    sh[2].zero_()
    e.rdp_kernel.fused_recovery_full_kv(sh, out, nd, S, T, n, 1, 2, -1)
    assert np.array_equal(sh.cpu().numpy(), want)
    assert np.array_equal(u16(out), np.concatenate([R.to_tn(kn).reshape(-1), R.to_tn(vn).reshape(-1)]))


@pytest.mark.parametrize("world,elems,star", [(8, 2048 * 128, 0), (4, 100, 3), (2, 8, 0), (8, 1000, 7), (3, 64, -4)])
def test_hook_ops_match_reference_math(rng, world, elems, star):
    e = pkg("ext")
    k_all, v_all = fp16_bits(rng, world * elems), fp16_bits(rng, world * elems)
    kt = torch.from_numpy(k_all).cuda().view(torch.float16)
    vt = torch.from_numpy(v_all).cuda().view(torch.float16)
    S = 2 * elems
    rows = torch.empty((world + 2, S), dtype=torch.uint16, device="cuda")
    for r in range(world):
        e.rdp_kv_ops.pack_row_from_block(kt[r * elems:(r + 1) * elems].view(1, 1, elems, 1),
                                         vt[r * elems:(r + 1) * elems].view(1, 1, elems, 1), rows, r)
    e.rdp_kv_ops.compute_rdp_parity(rows, nd=world, S=S, star_base=star)
    P, Q = R.hook_compute_parity(k_all, v_all, elems, star)
    got = rows.cpu().numpy()
    assert np.array_equal(got[world], P) and np.array_equal(got[world + 1], Q)


# ------------------------------------------------------------------ RS16 -----
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("k,m", [(8, 2), (4, 3), (6, 2), (3, 1), (5, 0)])
def test_rs16_dropin_matches_reference_math(rng, shape, k, m):
    rs = pkg("benchmark.rs.main")
    kn, vn, kt, vt = kv16(rng, shape)
    sh, meta = rs.forward_encode_kv(kt, vt, k, m)
    want, wmeta = R.rs16_forward_encode_kv(kn, vn, k, m)
    assert {kk: meta[kk] for kk in wmeta} == wmeta
    assert np.array_equal(sh.cpu().numpy(), want)
    pats = [list(c) for n in range(1, m + 1) for c in itertools.combinations(range(k + m), n)]
    for miss in pats[:40]:
        e = sh.clone()
        for i in miss:
            e[i].zero_()
        ko, vo = rs.backwards_decode_kv(e, meta, miss)
        assert np.array_equal(u16(ko), kn) and np.array_equal(u16(vo), vn), miss
        assert np.array_equal(e.cpu().numpy(), want), miss  # parity rows rebuilt too
        e2 = sh.clone()
        for i in miss:
            e2[i].zero_()
        want2 = want.copy()
        for i in miss:
            want2[i] = 0
        md = sorted(i for i in miss if i < k)
        mp = sorted(i - k for i in miss if i >= k)
        av = [p for p in range(m) if p not in mp]
        R.rs16_reconstruct(want2, k, md, av[:len(md)])
        rs.backwards_decode_kv(e2, meta, miss, rebuild_parity=False)
        assert np.array_equal(e2.cpu().numpy(), want2), miss  # the reference's exact end state


def test_rs16_errors(rng):
    rs = pkg("benchmark.rs.main")
    _, _, kt, vt = kv16(rng, (1, 1, 4, 8))
    sh, meta = rs.forward_encode_kv(kt, vt, 4, 1)
    with pytest.raises(RuntimeError, match="Not enough parity"):
        rs.backwards_decode_kv(sh, meta, [0, 1])


def test_rs16_ext_level(rng):
    e = pkg("ext")
    kn, vn, kt, vt = kv16(rng, (1, 2, 5, 8))
    N = kn.size
    out = torch.empty(2 * N, dtype=torch.uint16, device="cuda")
    e.rs_kernel.pack_fp16_pair_to_u16(kt, vt, out)
    kv = np.concatenate([kn.reshape(-1), vn.reshape(-1)])
    assert np.array_equal(out.cpu().numpy(), kv)
    k, m = 4, 2
    s = (2 * N + k - 1) // k
    dp = torch.zeros(k * s, dtype=torch.uint16, device="cuda")
    dp[:2 * N] = out
    sh = torch.empty((k + m, s), dtype=torch.uint16, device="cuda")
    e.rs_kernel.encode_rs_u16(dp, sh, k, m, s, None, None)
    want = R.rs16_encode(dp.cpu().numpy(), k, m, s)
    assert np.array_equal(sh.cpu().numpy(), want)
    sh[0].zero_()
    sh[3].zero_()
    e.rs_kernel.reconstruct_rs_u16_inplace(sh, s, k, m, torch.tensor([0, 3], dtype=torch.int32, device="cuda"),
                                           torch.tensor([0, 1], dtype=torch.int32, device="cuda"))
    assert np.array_equal(sh.cpu().numpy(), want)
    ko = torch.empty(N, dtype=torch.float16, device="cuda")
    vo = torch.empty(N, dtype=torch.float16, device="cuda")
    e.rs_kernel.u16_to_fp16_split(out, ko, vo, N, N)
    assert np.array_equal(u16(ko), kn.reshape(-1)) and np.array_equal(u16(vo), vn.reshape(-1))


# ----------------------------------------------- the reference itself, live --
@pytest.mark.parametrize("shape", [(1, 8, 256, 128), (1, 2, 7, 8)])
def test_live_reference_xor(rng, shape):
    ref = ref_mod("xor_kernel")
    x = pkg("benchmark.xor.main")
    _, _, kt, vt = kv16(rng, shape)
    B, H, T, D = shape
    n = B * H * D
    for k in (3, 8):
        kvb = torch.empty(4 * T * n, dtype=torch.uint8, device="cuda")
        ref.pack_kv(kt, vt, kvb, n, T)
        s, pad = x.determine_shard_size(kvb.numel(), k)
        dp = torch.zeros(k * s, dtype=torch.uint8, device="cuda")
        dp[:kvb.numel()] = kvb
        rsh = torch.zeros((k + 1, s), dtype=torch.uint8, device="cuda")
        ref.encode_xor(dp, rsh, k, s)
        torch.cuda.synchronize()
        ours = x.forward_encode_kv(kt, vt, k, 1)
        assert torch.equal(ours["shards_KV"].contiguous(), rsh)


@pytest.mark.parametrize("shape", [(1, 8, 512, 128), (1, 2, 7, 8)])
def test_live_reference_rdp(rng, shape):
    ref = ref_mod("rdp_kernel_rdp_parallel")
    r = pkg("benchmark.rdp.main")
    _, _, kt, vt = kv16(rng, shape)
    B, H, T, D = shape
    n = B * H * D
    for nd, star in ((8, 0), (6, 5)):
        S, _ = r.determine_shard_size_words(2 * T * n, nd)
        rsh = torch.zeros((nd + 2, S), dtype=torch.uint16, device="cuda")
        ktn = kt.permute(2, 0, 1, 3).contiguous().view(T, n)
        vtn = vt.permute(2, 0, 1, 3).contiguous().view(T, n)
        ref.fused_backup_full_kv(ktn, vtn, rsh, nd, S, T, n, star)
        torch.cuda.synchronize()
        ours = r.fused_backup_full_kv(kt, vt, nd, star_base=star)
        assert torch.equal(ours["shards_KV"].contiguous(), rsh)
        for a, b in ((1, -1), (0, 3)):
            x1 = rsh.clone()
            x1[a].zero_()
            out = torch.empty(2 * T * n, dtype=torch.float16, device="cuda")
            ref.fused_recovery_full_kv(x1, out, nd, S, T, n, star, a, b)
            torch.cuda.synchronize()
            ours["shards_KV"].copy_(rsh)
            ours["shards_KV"][a].zero_()
            ko, vo, _ = r.fused_recovery_full_kv(ours, a, b)
            assert torch.equal(ours["shards_KV"].contiguous(), x1)
            assert torch.equal(ko, out[:T * n].view(T, B, H, D).permute(1, 2, 0, 3))


def test_live_reference_rs16(rng):
    ref = ref_mod("rs_kernel16")
    rs = pkg("benchmark.rs.main")
    _, _, kt, vt = kv16(rng, (1, 8, 256, 128))
    ex, lg = rs.init_gf_tables()
    gexp = torch.from_numpy(ex).cuda()
    glog = torch.from_numpy(lg).cuda()
    for k, m in ((8, 2), (6, 3)):
        ours, meta = rs.forward_encode_kv(kt, vt, k, m)
        s = meta["shard_sz"]
        kv = torch.empty(meta["total"], dtype=torch.uint16, device="cuda")
        ref.pack_fp16_pair_to_u16(kt.reshape(-1), vt.reshape(-1), kv)
        dp = torch.zeros(k * s, dtype=torch.uint16, device="cuda")
        dp[:meta["total"]] = kv
        rsh = torch.empty((k + m, s), dtype=torch.uint16, device="cuda")
        ref.encode_rs_u16(dp, rsh, k, m, s, gexp, glog)
        torch.cuda.synchronize()
        assert torch.equal(ours.contiguous(), rsh)
        for miss in ([0, 1], [2, k], [k - 1]):
            md = [i for i in miss if i < k]
            x1 = rsh.clone()
            for i in miss:
                x1[i].zero_()
            mp = [i - k for i in miss if i >= k]
            av = [p for p in range(m) if p not in mp][:len(md)]
            ref.reconstruct_rs_u16_inplace(x1, s, k, m, torch.tensor(md, dtype=torch.int32, device="cuda"),
                                           torch.tensor(av, dtype=torch.int32, device="cuda"), gexp, glog)
            torch.cuda.synchronize()
            x2 = ours.clone()
            for i in miss:
                x2[i].zero_()
            rs.backwards_decode_kv(x2, meta, miss, rebuild_parity=False)
            assert torch.equal(x2.contiguous(), x1), miss


def test_live_reference_hook(rng):
    ref = ref_mod("rdp_kv_ops")
    e = pkg("ext")
    world, elems = 8, 2048 * 128
    k_all = torch.from_numpy(fp16_bits(rng, world * elems)).cuda().view(torch.float16)
    v_all = torch.from_numpy(fp16_bits(rng, world * elems)).cuda().view(torch.float16)
    S = 2 * elems
    r1 = torch.empty((world + 2, S), dtype=torch.uint16, device="cuda")
    r2 = torch.empty((world + 2, S), dtype=torch.uint16, device="cuda")
    for r in range(world):
        kb = k_all[r * elems:(r + 1) * elems].view(1, 1, elems, 1)
        vb = v_all[r * elems:(r + 1) * elems].view(1, 1, elems, 1)
        ref.pack_row_from_block(kb, vb, r1, r)
        e.rdp_kv_ops.pack_row_from_block(kb, vb, r2, r)
    ref.compute_rdp_parity(r1, nd=world, S=S, star_base=0)
    e.rdp_kv_ops.compute_rdp_parity(r2, nd=world, S=S, star_base=0)
    torch.cuda.synchronize()
    assert torch.equal(r1, r2)


# ------------------------------------------- unaligned caller layouts -------
# The reference's extension calls take [rows, S] tensors whose rows start at
# any byte offset; these sizes put every row (and the parity rows) at a
# different misalignment, large enough for the vector paths with ldu16 windows.
@pytest.mark.parametrize("s", [4793491, 200003, 65536 + 7])
@pytest.mark.parametrize("k", [2, 3, 7])
def test_unaligned_xor_extension_calls(rng, s, k):
    e = pkg("ext")
    dp_np = rng.integers(0, 256, k * s, dtype=np.uint8)
    dp = torch.from_numpy(dp_np).cuda()
    sh = torch.zeros((k + 1, s), dtype=torch.uint8, device="cuda")
    e.xor_kernel.encode_xor(dp, sh, k, s)
    want = R.xor_encode(dp_np, k, s)
    assert np.array_equal(sh.cpu().numpy(), want)
    miss = k // 2
    rec = torch.empty((1, s), dtype=torch.uint8, device="cuda")
    broken = sh.clone()
    broken[miss].zero_()
    e.xor_kernel.reconstruct_xor(broken, broken, rec, s, k, torch.tensor([miss], dtype=torch.int32, device="cuda"))
    assert torch.equal(broken, sh)


@pytest.mark.parametrize("nd,star", [(6, 0), (5, 3), (8, 1)])
@pytest.mark.parametrize("T,n", [(257, 40), (1024, 136)])
def test_unaligned_rdpref_extension_calls(rng, nd, star, T, n):
    e = pkg("ext")
    k_np, v_np = fp16_bits(rng, (T, n)), fp16_bits(rng, (T, n))
    S, _ = R.determine_shard_size_words(2 * T * n, nd)
    sh = torch.zeros((nd + 2, S), dtype=torch.uint16, device="cuda")  # rows 2*S bytes apart: any alignment
    kt = torch.from_numpy(k_np).cuda().view(torch.float16)
    vt = torch.from_numpy(v_np).cuda().view(torch.float16)
    e.rdp_kernel.fused_backup_full_kv(kt, vt, sh, nd, S, T, n, star)
    rows = R.rdpref_pack(k_np, v_np, nd, S)
    want = R.rdpref_parity(rows, nd, S, star)
    assert np.array_equal(sh.cpu().numpy(), want)
    out = torch.empty(2 * T * n, dtype=torch.float16, device="cuda")
    broken = sh.clone()
    broken[1].zero_()
    e.rdp_kernel.fused_recovery_full_kv(broken, out, nd, S, T, n, star, 1, -1)
    assert np.array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16),
                          np.concatenate([k_np.reshape(-1), v_np.reshape(-1)]))


@pytest.mark.parametrize("k,m,s", [(6, 2, 100003), (3, 3, 65536 + 5), (8, 2, 4099)])
def test_unaligned_rs16_extension_calls(rng, k, m, s):
    e = pkg("ext")
    dp_np = rng.integers(0, 1 << 16, k * s, dtype=np.uint16)
    sh = torch.zeros((k + m, s), dtype=torch.uint16, device="cuda")
    e.rs_kernel.encode_rs_u16(torch.from_numpy(dp_np).cuda(), sh, k, m, s)
    assert np.array_equal(sh.cpu().numpy(), R.rs16_encode(dp_np, k, m, s))


@pytest.mark.parametrize("B,H,T,D", [(1, 3, 129, 40), (2, 2, 300, 128), (1, 1, 1000, 12)])
def test_unaligned_bhtd_layouts(rng, B, H, T, D):
    r = pkg("benchmark.rdp.main")
    k_np, v_np = fp16_bits(rng, (B, H, T, D)), fp16_bits(rng, (B, H, T, D))
    kt = torch.from_numpy(k_np).cuda().view(torch.float16)
    vt = torch.from_numpy(v_np).cuda().view(torch.float16)
    for nd in (5, 7):
        p = r.fused_backup_full_kv(kt, vt, nd, star_base=2)
        enc, S, _ = R.rdpref_backup(k_np, v_np, nd, 2)
        assert np.array_equal(u16(p["shards_KV"]), enc)
        ko, vo, _ = r.fused_recovery_full_kv(p, 2)
        assert np.array_equal(u16(ko), k_np) and np.array_equal(u16(vo), v_np)
