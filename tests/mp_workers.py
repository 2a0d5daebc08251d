"""Worker functions for multi-process tests (importable by spawned children)."""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _init(rank, world, port, backend="gloo"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if backend == "nccl":
        import datetime

        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
    else:
        dist.init_process_group("gloo", rank=rank, world_size=world)


def _pkg(sub=""):
    import importlib

    return importlib.import_module("26mlsys-ae-ghostserve_b200" + ("." + sub if sub else ""))


# ------------------------------------------------------------- CPU (gloo) ----
def chunk_ids(rank, world, port, mode, out):
    _init(rank, world, port)
    hook = _pkg("hook")
    ft = hook.KVFaultTolerance(hook.HookConfig(mode=mode, metrics_file=None))
    ids = [ft.next_chunk_id(device=None) for _ in range(5)]
    out.put((rank, ids))
    dist.destroy_process_group()


def gather(rank, world, port, out):
    _init(rank, world, port)
    hook = _pkg("hook")
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="reference", metrics_file=None))
    k = torch.full((3, 1, 4), rank, dtype=torch.float16)
    v = torch.full((3, 1, 4), 10 + rank, dtype=torch.float16)
    for dst in range(world):
        res = ft.gather_kv(k, v, dst)
        if rank == dst:
            k_all, v_all, elems = res
            out.put((rank, dst, elems, k_all.tolist(), v_all.tolist()))
        else:
            assert res is None
    dist.destroy_process_group()


def peer_table(rank, world, port, out):
    _init(rank, world, port)
    p2p = _pkg("p2p")
    bufs = [torch.zeros(16 * (j + 1), dtype=torch.uint8) for j in range(3)]
    exporter = lambda t: (bytes([rank]) * 64, t.numel())  # noqa: E731  (fake handle: owner rank)
    importer = lambda h, off: 1000 * h[0] + off  # noqa: E731
    grp = p2p.PeerGroup.create(bufs, exporter=exporter, importer=importer, closer=lambda: None)
    out.put((rank, grp.table))
    grp.close()
    dist.destroy_process_group()


# ----------------------------------------------- GPU (2 processes, 1 GPU) ----
def ipc_sliced_encode(rank, world, port, scheme, out):
    """Each rank stages a KV shard in IPC-shared memory; every rank encodes its
    stripe slice reading all shards through mapped pointers; rank 0 assembles
    the slices and checks them against the oracle."""
    _init(rank, world, port)
    torch.cuda.set_device(0)
    g = _pkg()
    p2p = _pkg("p2p")
    from oracle import codes

    rng = np.random.default_rng(100 + rank)
    half = 16 * 1000 + 4096
    k_host = rng.integers(0, 256, half, dtype=np.uint8)
    v_host = rng.integers(0, 256, half, dtype=np.uint8)
    kt = torch.from_numpy(k_host).cuda()
    vt = torch.from_numpy(v_host).cuda()
    grp = p2p.PeerGroup.create([kt, vt])
    torch.cuda.synchronize()
    dist.barrier()
    spec = {"rdp": g.CodeSpec.rdp(world, unit=256), "xor": g.CodeSpec.xor(world), "rs8": g.CodeSpec.rs8(world, 2)}[
        scheme]
    data_bytes = 2 * half
    pb = spec.parity_bytes(data_bytes)
    gran = spec.stripe_bytes()
    lo, hi = p2p.stripe_slice(rank, world, pb // gran)
    lo, hi = lo * gran, hi * gran
    par = [torch.zeros(max(hi - lo, 16), dtype=torch.uint8, device="cuda") for _ in range(spec.m)]
    g.codec.encode_ptrs(spec, [grp.ptr(r, 0) for r in range(world)], [grp.ptr(r, 1) for r in range(world)], half,
                        data_bytes, [t.data_ptr() - lo for t in par], lo, hi)
    torch.cuda.synchronize()
    mine = [t[:hi - lo].cpu() for t in par]
    kv = torch.from_numpy(np.concatenate([k_host, v_host]))
    all_kv = [torch.empty_like(kv) for _ in range(world)]
    dist.all_gather(all_kv, kv)
    sizes = [None] * world
    dist.all_gather_object(sizes, (lo, hi))
    slices = [None] * world
    dist.all_gather_object(slices, [m.numpy() for m in mine])
    ok = True
    if rank == 0:
        data = [a.numpy() for a in all_kv]
        if scheme == "rdp":
            want = codes.rdp_encode(data, spec.p, spec.unit)
        elif scheme == "xor":
            want = [codes.xor_encode(data)]
        else:
            want = codes.rs8_encode(data, 2)
        for j in range(spec.m):
            got = np.concatenate([slices[r][j] for r in range(world)])
            ok = ok and np.array_equal(got, want[j])
    dist.barrier()
    grp.close()
    out.put((rank, ok))
    dist.destroy_process_group()


def hook_fused(rank, world, port, backend, unit, out):
    """The hook's fused mode end to end: gloo = ranks sharing cuda:0 (CUDA IPC
    within one device), nccl = one GPU per rank (NVLink peer reads)."""
    _init(rank, world, port, backend)
    dev = rank if backend == "nccl" else 0
    torch.cuda.set_device(dev)
    hook = _pkg("hook")
    from oracle import codes

    ft = hook.KVFaultTolerance(hook.HookConfig(mode="fused", scheme="rdp", unit=unit, metrics_file=None))
    rng = np.random.default_rng(7 + rank)
    ok = True
    for step in range(3):
        tokens = 64 + 32 * step
        k = torch.from_numpy(rng.standard_normal((tokens, 1, 128)).astype(np.float32)).cuda().to(torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((tokens, 1, 128)).astype(np.float32)).cuda().to(torch.bfloat16)
        par, (lo, hi) = ft.encode_chunk(k, v, step + 1)
        torch.cuda.synchronize()
        shard = torch.cat([k.view(torch.uint8).reshape(-1), v.view(torch.uint8).reshape(-1)]).cpu().numpy()
        shards = [None] * world
        dist.all_gather_object(shards, shard)
        got = [None] * world
        dist.all_gather_object(got, [p.cpu().numpy() for p in par])
        if rank == 0:
            spec = ft._spec(world)
            want = codes.rdp_encode(list(shards), spec.p, spec.unit)
            for j in range(2):
                ok = ok and np.array_equal(np.concatenate([got[r][j] for r in range(world)]), want[j])
    ft.close()
    recs = [r["chunk_id"] for r in ft.records]
    out.put((rank, ok, recs))
    dist.destroy_process_group()


def hook_recover(rank, world, port, backend, scheme, lost_sets, out):
    """Encode several prefill chunks of a layer-major KV cache through the hook,
    then lose ranks (their chunk KV zeroed, as on a replacement GPU) and rebuild
    it with KVFaultTolerance.recover_parts; every rebuilt byte must match."""
    _init(rank, world, port, backend)
    dev = rank if backend == "nccl" else 0
    torch.cuda.set_device(dev)
    hook = _pkg("hook")
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="fused", scheme=scheme, unit=512, host_keep=4,
                                               metrics_file=None))
    layers, hk, tmax, d = 3, 2, 256, 64
    gen = torch.Generator(device="cuda").manual_seed(11 + rank)
    kc = torch.randn(layers, hk, tmax, d, device="cuda", generator=gen).to(torch.bfloat16)
    vc = torch.randn(layers, hk, tmax, d, device="cuda", generator=gen).to(torch.bfloat16)

    def parts(pos0, t):
        return ([kc[li, :, pos0:pos0 + t] for li in range(layers)],
                [vc[li, :, pos0:pos0 + t] for li in range(layers)])

    chunks = [(c + 1, 40 * c, 40) for c in range(6)]
    for cid, pos0, t in chunks:
        ft.encode_parts(*parts(pos0, t), cid)
    ft.encode_parts(*parts(200, 40), 6)  # an id encoded again keeps one store slot
    ft.flush()
    ok = True
    for lost in lost_sets:
        for cid, pos0, t in chunks[2:]:
            pk, pv = parts(pos0, t)
            want = [x.clone() for x in pk + pv]
            if rank in lost:
                for x in pk + pv:
                    x.fill_(0)
            ft.recover_parts(cid, lost, pk, pv)
            torch.cuda.synchronize()
            ok = ok and all(torch.equal(a, b) for a, b in zip(pk + pv, want))
    evicted = True
    try:
        ft.recover_parts(1, lost_sets[0], *parts(0, 40))
        evicted = False
    except KeyError:
        pass
    ft.close()
    oks = [None] * world
    dist.all_gather_object(oks, ok)
    out.put((rank, all(oks), evicted))
    dist.destroy_process_group()


def hook_pool(rank, world, port, backend, out):
    """The hook as SGLang drives it: a FlashInfer-like backend whose KV pool
    [slots, 2, heads, 128] is read through each extend call's slot_mapping
    (a permutation with -1 padding). Fused parity must equal the oracle's over
    the gathered rows (zero rows for -1), and a lost rank's pool rows must come
    back bit-exact through recover_pool."""
    _init(rank, world, port, backend)
    dev = rank if backend == "nccl" else 0
    torch.cuda.set_device(dev)
    hook = _pkg("hook")
    from oracle import codes

    class FlashInferAttnBackend:
        def __init__(self):
            g = torch.Generator(device="cuda").manual_seed(100 + rank)
            self.kv_buffer = torch.randn(512, 2, 2, 128, device="cuda", generator=g).to(torch.bfloat16)

        def forward_extend(self, batch, layer=None, save_kv_cache=True):
            return "attn-out"

    class Batch:
        def __init__(self, slot_mapping):
            self.slot_mapping = slot_mapping

    be = FlashInferAttnBackend()
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="fused", scheme="rdp", unit=1024, metrics_file=None))
    assert hook.patch_backend(be, ft)
    gen = torch.Generator().manual_seed(5)  # same slot lists on every rank, as tensor-parallel ranks see
    calls = []
    for n, dtype in ((96, torch.int64), (40, torch.int32), (200, torch.int64)):
        perm = torch.randperm(512, generator=gen)[:n].to(dtype)
        perm[torch.randperm(n, generator=gen)[: n // 8]] = -1
        calls.append(perm.cuda())
    ok = True
    spec = ft._spec(world)
    for sm in calls:
        assert be.forward_extend(Batch(sm), layer=0) == "attn-out"
        torch.cuda.synchronize()
        s64 = sm.to(torch.int64)
        rows = be.kv_buffer[s64.clamp(min=0)].clone()
        rows[s64 < 0] = 0
        shard = torch.cat([rows[:, 0].reshape(-1).view(torch.uint8), rows[:, 1].reshape(-1).view(torch.uint8)])
        shards = [None] * world
        dist.all_gather_object(shards, shard.cpu().numpy())
        ft.flush()
        entry = ft._store[ft.chunk_counter]
        mine = entry["host"].numpy().copy()
        got = [None] * world
        dist.all_gather_object(got, (entry["lo"], entry["hi"], mine))
        if rank == 0:
            want = codes.rdp_encode(list(shards), spec.p, spec.unit)
            for j in range(2):
                parts = [g[2][j * (g[1] - g[0]):(j + 1) * (g[1] - g[0])] for g in got]
                ok = ok and np.array_equal(np.concatenate(parts), want[j])
    # lose rank 1 (and both ranks) and rebuild every call's rows in the pool
    for lost in ([1], [0, 1]):
        saved = be.kv_buffer.clone()
        for cid, sm in enumerate(calls, start=1):
            if rank in lost:
                s64 = sm.to(torch.int64)
                be.kv_buffer[s64[s64 >= 0]] = 0
            ft.recover_pool(cid, lost, be.kv_buffer, sm)
        torch.cuda.synchronize()
        ok = ok and torch.equal(be.kv_buffer, saved)
    ft.close()
    oks = [None] * world
    dist.all_gather_object(oks, ok)
    out.put((rank, all(oks), [r["chunk_id"] for r in ft.records]))
    dist.destroy_process_group()


def hook_reference(rank, world, port, backend, out):
    """The hook in mode="reference" as SGLang drives it: a FlashInfer-like
    backend's extend calls go through on_extend (active slots, chunk-id
    broadcast, NCCL gather to the rotating rank, fp16 cast, pack, mod-S parity,
    host copy). The destination rank's P/Q must equal what the reference's own
    rdp_kv_ops extension computes from the same gathered rows."""
    _init(rank, world, port, backend)
    torch.cuda.set_device(rank)
    hook = _pkg("hook")
    from oracle import build_ref

    if not build_ref.built("rdp_kv_ops"):
        out.put((rank, "skip", []))
        dist.destroy_process_group()
        return
    ref = build_ref.load_ref("rdp_kv_ops")

    class FlashInferAttnBackend:
        def __init__(self):
            g = torch.Generator(device="cuda").manual_seed(200 + rank)
            self.kv_buffer = torch.randn(512, 2, 1, 128, device="cuda", generator=g).to(torch.bfloat16)

        def forward_extend(self, batch, layer=None, save_kv_cache=True):
            return "attn-out"

    class Batch:
        def __init__(self, slot_mapping):
            self.slot_mapping = slot_mapping

    be = FlashInferAttnBackend()
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="reference", star_base=1, metrics_file=None))
    seen = []
    real = ft.compute_parity_to_cpu

    def capture(K_all, V_all, elems, chunk_id, dst_rank):
        P, Q = real(K_all, V_all, elems, chunk_id, dst_rank)
        seen.append((K_all.clone(), V_all.clone(), elems, P, Q))
        return P, Q

    ft.compute_parity_to_cpu = capture
    assert hook.patch_backend(be, ft)
    gen = torch.Generator().manual_seed(9)  # the same slot lists on every rank
    ok = True
    for n in (64, 40, 200):
        perm = torch.randperm(512, generator=gen)[:n]
        perm[torch.randperm(n, generator=gen)[: n // 8]] = -1
        assert be.forward_extend(Batch(perm.cuda()), layer=0) == "attn-out"
        torch.cuda.synchronize()
    for K_all, V_all, elems, P, Q in seen:
        S = 2 * elems
        rows = torch.empty((world + 2, S), dtype=torch.uint16, device="cuda")
        for r in range(world):
            k = K_all.narrow(0, r * elems, elems).to(torch.float16)
            v = V_all.narrow(0, r * elems, elems).to(torch.float16)
            ref.pack_row_from_block(k.view(1, 1, elems, 1), v.view(1, 1, elems, 1), rows, r)
        ref.compute_rdp_parity(rows, nd=world, S=S, star_base=1)
        torch.cuda.synchronize()
        ok = ok and torch.equal(rows[world].cpu(), P) and torch.equal(rows[world + 1].cpu(), Q)
    # the gathered rows are the active slots' K and V of every rank, in rank order
    recs = [(r["chunk_id"], r["dst_rank"]) for r in ft.records]
    ft.close()
    oks = [None] * world
    dist.all_gather_object(oks, (ok, len(seen)))
    out.put((rank, oks, recs))
    dist.destroy_process_group()


def chunk_mode_calls(rank, world, port, out):
    """protect="chunk" on the host: the hook encodes once per chunk_layers
    extend calls, with that chunk's pools in call order (encode_pools mocked)."""
    _init(rank, world, port)
    hook = _pkg("hook")
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="fused", protect="chunk", chunk_layers=3, metrics_file=None))
    got = []
    ft.encode_pools = lambda pools, slots, cid: got.append(([int(p[0, 0, 0, 0]) for p in pools], cid,
                                                            slots.tolist()))

    class Batch:
        def __init__(self, sm):
            self.slot_mapping = sm

    pools = [torch.full((8, 2, 1, 8), float(li)) for li in range(3)]
    for c in range(2):
        sm = torch.arange(4) + 4 * c
        for li in range(3):
            ft.on_extend(Batch(sm), pools[li])
    out.put((rank, got))
    dist.destroy_process_group()


def hook_pool_chunk(rank, world, port, backend, out):
    """protect="chunk" on the GPU: three layers' pools (one per extend call of
    a chunk) are encoded as one codeword per chunk whose data shard is the row
    stream [layer 0 K, layer 0 V, layer 1 K, ...]; parity must equal the
    oracle's, and recover_pool with the list of pools must bring a lost rank's
    rows back bit-exact in every layer."""
    _init(rank, world, port, backend)
    dev = rank if backend == "nccl" else 0
    torch.cuda.set_device(dev)
    hook = _pkg("hook")
    from oracle import codes

    L = 3
    g = torch.Generator(device="cuda").manual_seed(300 + rank)
    pools = [torch.randn(256, 2, 2, 64, device="cuda", generator=g).to(torch.bfloat16) for _ in range(L)]

    class FlashInferAttnBackend:
        kv_buffer = None

        def forward_extend(self, batch, layer=None, save_kv_cache=True):
            return "attn-out"

    class Batch:
        def __init__(self, slot_mapping):
            self.slot_mapping = slot_mapping

    be = FlashInferAttnBackend()
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="fused", scheme="rdp", unit=1024, protect="chunk",
                                               chunk_layers=L, metrics_file=None))
    assert hook.patch_backend(be, ft)
    gen = torch.Generator().manual_seed(6)
    calls = []
    for n in (64, 24):
        perm = torch.randperm(256, generator=gen)[:n]
        perm[torch.randperm(n, generator=gen)[: n // 8]] = -1
        calls.append(perm.cuda())
    ok = True
    spec = ft._spec(world)
    for sm in calls:
        for li in range(L):
            be.kv_buffer = pools[li]
            assert be.forward_extend(Batch(sm), layer=li) == "attn-out"
        torch.cuda.synchronize()
        s64 = sm.to(torch.int64)
        parts = []
        for p in pools:
            rows = p[s64.clamp(min=0)].clone()
            rows[s64 < 0] = 0
            parts += [rows[:, 0].reshape(-1).view(torch.uint8), rows[:, 1].reshape(-1).view(torch.uint8)]
        shard = torch.cat(parts)
        shards = [None] * world
        dist.all_gather_object(shards, shard.cpu().numpy())
        ft.flush()
        entry = ft._store[ft.chunk_counter]
        mine = entry["host"].numpy().copy()
        got = [None] * world
        dist.all_gather_object(got, (entry["lo"], entry["hi"], mine))
        if rank == 0:
            want = codes.rdp_encode(list(shards), spec.p, spec.unit)
            for j in range(2):
                sl = [x[2][j * (x[1] - x[0]):(j + 1) * (x[1] - x[0])] for x in got]
                ok = ok and np.array_equal(np.concatenate(sl), want[j])
    for lost in ([1], [0, 1]) if world > 1 else ([0],):
        saved = [p.clone() for p in pools]
        for cid, sm in enumerate(calls, start=1):
            if rank in lost:
                s64 = sm.to(torch.int64)
                for p in pools:
                    p[s64[s64 >= 0]] = 0
            ft.recover_pool(cid, lost, pools, sm)
        torch.cuda.synchronize()
        ok = ok and all(torch.equal(p, q) for p, q in zip(pools, saved))
    ft.close()
    oks = [None] * world
    dist.all_gather_object(oks, ok)
    out.put((rank, all(oks), [r["chunk_id"] for r in ft.records]))
    dist.destroy_process_group()
