"""Time the reference's own CUDA kernels (built from its sources into
oracle/_ref) against this engine's drop-ins for the same extension calls, on
the same bytes, on one GPU. Each pair computes the same function (checked
bit-exact here too), so the ratio is kernel speed only.

    python tests/ref_speed.py          # prints one JSON object

Used by tests/test_gpu_ref_speed.py at a smaller size."""
from __future__ import annotations

import importlib
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

from oracle import build_ref  # noqa: E402

PKG = "26mlsys-ae-ghostserve_b200"


def _time(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3  # us


def _graph_time(fn, reps: int) -> float:
    """Per-call device time of reps calls replayed from one CUDA graph (us)."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3


def measure(T: int = 2048, n: int = 4096, reps: int = 20) -> dict:
    """KV of one rank's chunk: K and V fp16 [T tokens, n = layers x heads x dim]."""
    ext = importlib.import_module(PKG + ".ext")
    gen = torch.Generator(device="cuda").manual_seed(0)
    out = {"T": T, "n": n}

    def rnd16(*shape):
        return torch.randint(0, 1 << 16, shape, generator=gen, device="cuda", dtype=torch.int32).to(
            torch.int16).view(torch.float16)

    kt, vt = rnd16(T, n), rnd16(T, n)  # token-major K/V words
    kv_bytes = 4 * T * n

    # XOR: encode_xor(data_padded, shards, k, s) -- data rows copied + parity row
    if build_ref.built("xor_kernel"):
        ref = build_ref.load_ref("xor_kernel")
        k = 7
        s = -(-kv_bytes // k)
        dp = torch.zeros(k * s, dtype=torch.uint8, device="cuda")
        dp[:kv_bytes] = torch.cat([kt.reshape(-1), vt.reshape(-1)]).view(torch.uint8)
        a = torch.zeros((k + 1, s), dtype=torch.uint8, device="cuda")
        b = torch.zeros((k + 1, s), dtype=torch.uint8, device="cuda")
        tr = _time(lambda: ref.encode_xor(dp, a, k, s), reps)
        to = _time(lambda: ext.xor_kernel.encode_xor(dp, b, k, s), reps)
        out["xor_encode_xor"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1), "speedup": round(tr / to, 2),
                                 "equal": bool(torch.equal(a, b)), "bytes": (2 * k + 1) * s}

    # mod-S RDP backup: fused_backup_full_kv(K_TN, V_TN, shards, nd, S, T, n, star)
    if build_ref.built("rdp_kernel_rdp_parallel"):
        ref = build_ref.load_ref("rdp_kernel_rdp_parallel")
        nd = 6
        S = -(-(2 * T * n) // nd)
        a = torch.zeros((nd + 2, S), dtype=torch.uint16, device="cuda")
        b = torch.zeros((nd + 2, S), dtype=torch.uint16, device="cuda")
        tr = _time(lambda: ref.fused_backup_full_kv(kt, vt, a, nd, S, T, n, 0), reps)
        to = _time(lambda: ext.rdp_kernel.fused_backup_full_kv(kt, vt, b, nd, S, T, n, 0), reps)
        out["rdpref_fused_backup_full_kv"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1),
                                              "speedup": round(tr / to, 2), "equal": bool(torch.equal(a, b)),
                                              "bytes": 4 * T * n + (nd + 2) * S * 2}
        # single-row recovery (data row 2 lost) back to the token-major output
        outa = torch.empty(2 * T * n, dtype=torch.float16, device="cuda")
        outb = torch.empty(2 * T * n, dtype=torch.float16, device="cuda")
        tr = _time(lambda: ref.fused_recovery_full_kv(a, outa, nd, S, T, n, 0, 2, -1), reps)
        to = _time(lambda: ext.rdp_kernel.fused_recovery_full_kv(b, outb, nd, S, T, n, 0, 2, -1), reps)
        out["rdpref_fused_recovery_full_kv"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1),
                                                "speedup": round(tr / to, 2),
                                                "equal": bool(torch.equal(outa.view(torch.int16),
                                                                          outb.view(torch.int16)))}

    # RS over GF(2^16): encode_rs_u16(data_padded, shards, k, m, s, gf_exp, gf_log)
    if build_ref.built("rs_kernel16"):
        ref = build_ref.load_ref("rs_kernel16")
        rs = importlib.import_module(PKG + ".benchmark.rs.main")
        ex, lg = rs.init_gf_tables()
        gexp, glog = torch.from_numpy(ex).cuda(), torch.from_numpy(lg).cuda()
        k, m = 6, 2
        total = 2 * T * n
        s = -(-total // k)
        dp = torch.zeros(k * s, dtype=torch.uint16, device="cuda")
        dp[:total] = torch.cat([kt.reshape(-1), vt.reshape(-1)]).view(torch.uint16)
        a = torch.zeros((k + m, s), dtype=torch.uint16, device="cuda")
        b = torch.zeros((k + m, s), dtype=torch.uint16, device="cuda")
        tr = _time(lambda: ref.encode_rs_u16(dp, a, k, m, s, gexp, glog), reps)
        to = _time(lambda: ext.rs_kernel.encode_rs_u16(dp, b, k, m, s, gexp, glog), reps)
        out["rs16_encode_rs_u16"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1), "speedup": round(tr / to, 2),
                                     "equal": bool(torch.equal(a, b)), "bytes": (2 * k + m) * s * 2}

    # the hook's parity: compute_rdp_parity(rows, nd, S, star) over world = 8 rows
    if build_ref.built("rdp_kv_ops"):
        ref = build_ref.load_ref("rdp_kv_ops")
        world, elems = 8, T * n // 8
        S = 2 * elems
        src = torch.randint(0, 1 << 16, (world + 2, S), generator=gen, device="cuda", dtype=torch.int32).to(
            torch.int16).view(torch.uint16)
        a, b = src.clone(), src.clone()
        tr = _time(lambda: ref.compute_rdp_parity(a, nd=world, S=S, star_base=0), reps)
        to = _time(lambda: ext.rdp_kv_ops.compute_rdp_parity(b, nd=world, S=S, star_base=0), reps)
        # both launch on the current stream, so both can be replayed from a graph: device time alone
        gr = _graph_time(lambda: ref.compute_rdp_parity(a, nd=world, S=S, star_base=0), reps)
        go = _graph_time(lambda: ext.rdp_kv_ops.compute_rdp_parity(b, nd=world, S=S, star_base=0), reps)
        out["hook_compute_rdp_parity"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1),
                                          "speedup": round(tr / to, 2), "equal": bool(torch.equal(a, b)),
                                          "bytes": (world + 2) * S * 2, "ref_device_us": round(gr, 1),
                                          "ours_device_us": round(go, 1), "device_speedup": round(gr / go, 2)}
    out.update(measure_flows(T, n, reps))
    return out


def measure_flows(T: int, n: int, reps: int) -> dict:
    """The Python entry points: the reference's GPU call sequence (its
    extension calls and tensor ops as benchmark/{xor,rdp,rs}/main.py issue
    them, minus host-side prints and the per-call Python GF-table build of
    rs/main.py, here built once) against this package's drop-in functions."""
    xm = importlib.import_module(PKG + ".benchmark.xor.main")
    rm = importlib.import_module(PKG + ".benchmark.rdp.main")
    sm = importlib.import_module(PKG + ".benchmark.rs.main")
    gen = torch.Generator(device="cuda").manual_seed(1)
    B, H, D = 1, n // 128, 128
    keys = torch.randint(0, 1 << 16, (B, H, T, D), generator=gen, device="cuda", dtype=torch.int32).to(
        torch.int16).view(torch.float16)
    values = torch.randint(0, 1 << 16, (B, H, T, D), generator=gen, device="cuda", dtype=torch.int32).to(
        torch.int16).view(torch.float16)
    out = {}
    if build_ref.built("xor_kernel"):
        ref = build_ref.load_ref("xor_kernel")
        k = 7

        def ref_xor():  # xor/main.py:47-113
            kv = torch.empty(4 * T * n, dtype=torch.uint8, device="cuda")
            ref.pack_kv(keys, values, kv, n, T)
            s, _ = xm.determine_shard_size(kv.numel(), k)
            dp = torch.zeros(k * s, dtype=torch.uint8, device="cuda")
            dp[:kv.numel()] = kv
            sh = torch.zeros((k + 1, s), dtype=torch.uint8, device="cuda")
            ref.encode_xor(dp, sh, k, s)
            return sh

        tr = _time(ref_xor, reps)
        to = _time(lambda: xm.forward_encode_kv(keys, values, k, 1), reps)
        eq = torch.equal(ref_xor(), xm.forward_encode_kv(keys, values, k, 1)["shards_KV"])
        out["flow_xor_forward_encode_kv"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1),
                                             "speedup": round(tr / to, 2), "equal": bool(eq)}
    if build_ref.built("rdp_kernel_rdp_parallel"):
        ref = build_ref.load_ref("rdp_kernel_rdp_parallel")
        nd = 6

        def ref_rdp():  # rdp/main.py:44-92, with its two synchronizations around the timed kernel
            ktn = keys.permute(2, 0, 1, 3).contiguous().view(T, n)
            vtn = values.permute(2, 0, 1, 3).contiguous().view(T, n)
            S, _ = rm.determine_shard_size_words(2 * T * n, nd)
            sh = torch.zeros((nd + 2, S), dtype=torch.uint16, device="cuda")
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(True), torch.cuda.Event(True)
            t0.record()
            ref.fused_backup_full_kv(ktn, vtn, sh, nd, S, T, n, 0)
            t1.record()
            torch.cuda.synchronize()
            return sh

        tr = _time(ref_rdp, reps)
        to = _time(lambda: rm.fused_backup_full_kv(keys, values, nd), reps)
        eq = torch.equal(ref_rdp(), rm.fused_backup_full_kv(keys, values, nd)["shards_KV"])
        out["flow_rdp_fused_backup_full_kv"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1),
                                                "speedup": round(tr / to, 2), "equal": bool(eq)}
    if build_ref.built("rs_kernel16"):
        ref = build_ref.load_ref("rs_kernel16")
        ex, lg = sm.init_gf_tables()
        gexp, glog = torch.from_numpy(ex).cuda(), torch.from_numpy(lg).cuda()
        k, m = 6, 2

        def ref_rs():  # rs/main.py:57-137 (tables built once, not per call)
            tot = keys.numel() + values.numel()
            kv = torch.empty(tot, dtype=torch.uint16, device="cuda")
            ref.pack_fp16_pair_to_u16(keys.contiguous().view(-1), values.contiguous().view(-1), kv)
            s, pad = sm.shard_size_and_pad(tot, k)
            dp = torch.empty(k * s, dtype=torch.uint16, device="cuda")
            if pad:
                dp.fill_(0)
            dp[:tot].copy_(kv)
            sh = torch.empty((k + m, s), dtype=torch.uint16, device="cuda")
            ref.encode_rs_u16(dp, sh, k, m, s, gexp, glog)
            return sh

        tr = _time(ref_rs, reps)
        to = _time(lambda: sm.forward_encode_kv(keys, values, k, m), reps)
        eq = torch.equal(ref_rs(), sm.forward_encode_kv(keys, values, k, m)[0])
        out["flow_rs_forward_encode_kv"] = {"ref_us": round(tr, 1), "ours_us": round(to, 1),
                                            "speedup": round(tr / to, 2), "equal": bool(eq)}
    return out


if __name__ == "__main__":
    print(json.dumps({"config_3_layer_call": measure(T=1024, n=2048), "full_chunk": measure()}), flush=True)
