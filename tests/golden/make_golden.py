"""Generate golden vectors from the reference's own CUDA extensions.

    python tests/golden/make_golden.py [outdir]     (on a GPU box)

Runs the reference extensions compiled from the reference sources by
oracle/build_ref.py (oracle/_ref/*) on small seeded inputs generated on the
host, and writes inputs and outputs to ``ref_*.npz``.  tests/test_golden.py
checks the CPU oracle (oracle/reference.py) against these files, which pins the
oracle to the reference's actual behaviour.  Inputs are bf16 N(0,1) bit
patterns (the KV dtype of the benchmark configs) handed to the reference as
fp16 by bit reinterpretation, plus fp16 N(0,1) for the RS case.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def bf16_bits(rng, shape):
    x = rng.standard_normal(shape, dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def main(out_dir: str = HERE) -> None:
    import torch

    from oracle.build_ref import load_ref

    dev = torch.device("cuda")

    def t16(a):  # uint16 bit patterns -> fp16 CUDA tensor (bit reinterpretation)
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev).view(torch.float16)

    rng = np.random.default_rng(20261201)

    # ------------------------------------------------------------------ XOR --
    xk = load_ref("xor_kernel")
    xor = {}
    for case, (shape, k, miss) in enumerate([((1, 2, 16, 8), 3, 1), ((1, 2, 16, 8), 8, 8), ((1, 3, 5, 8), 7, 0)]):
        kb, vb = bf16_bits(rng, shape), bf16_bits(rng, shape)
        B, H, T, D = shape
        n = B * H * D
        kvb = torch.empty(4 * T * n, dtype=torch.uint8, device=dev)
        xk.pack_kv(t16(kb), t16(vb), kvb, n, T)
        s = (kvb.numel() + k - 1) // k
        dp = torch.zeros(k * s, dtype=torch.uint8, device=dev)
        dp[:kvb.numel()] = kvb
        sh = torch.zeros((k + 1, s), dtype=torch.uint8, device=dev)
        xk.encode_xor(dp, sh, k, s)
        enc = sh.cpu().numpy().copy()
        sh[miss].zero_()
        rec = torch.empty((1, s), dtype=torch.uint8, device=dev)
        xk.reconstruct_xor(sh, sh, rec, s, k, torch.tensor([miss], dtype=torch.int32, device=dev))
        out = torch.empty(2 * T * n, dtype=torch.float16, device=dev)
        xk.unpack_kv(sh[:k].contiguous().view(-1), out, n, T)
        torch.cuda.synchronize()
        p = f"c{case}_"
        xor.update({p + "keys": kb, p + "values": vb, p + "shape": np.array(shape), p + "k": np.array(k),
                    p + "miss": np.array(miss), p + "kv_bytes": kvb.cpu().numpy(), p + "encoded": enc,
                    p + "rebuilt": sh.cpu().numpy(), p + "recovered": rec.cpu().numpy(),
                    p + "unpacked": out.view(torch.uint16).cpu().numpy()})
    np.savez_compressed(os.path.join(out_dir, "ref_xor.npz"), **xor)

    # ------------------------------------------------------------ RDP (ref) --
    rk = load_ref("rdp_kernel_rdp_parallel")
    rdp = {}
    cases = [((1, 2, 12, 8), 4, 0, 1, -1), ((1, 2, 12, 8), 8, 3, 2, 5), ((2, 1, 9, 8), 5, 1, 4, -1),
             ((1, 2, 12, 8), 6, 2, 0, 3)]
    for case, (shape, nd, star, a, b) in enumerate(cases):
        kb, vb = bf16_bits(rng, shape), bf16_bits(rng, shape)
        B, H, T, D = shape
        n = B * H * D
        S = (2 * T * n + nd - 1) // nd
        sh = torch.zeros((nd + 2, S), dtype=torch.uint16, device=dev)
        ktn = t16(kb).permute(2, 0, 1, 3).contiguous().view(T, n)
        vtn = t16(vb).permute(2, 0, 1, 3).contiguous().view(T, n)
        rk.fused_backup_full_kv(ktn, vtn, sh, nd, S, T, n, star)
        enc = sh.cpu().numpy().copy()
        if b < 0:
            sh[a].zero_()  # a real single erasure
        out = torch.empty(2 * T * n, dtype=torch.float16, device=dev)
        rk.fused_recovery_full_kv(sh, out, nd, S, T, n, star, a, b)
        torch.cuda.synchronize()
        p = f"c{case}_"
        rdp.update({p + "keys": kb, p + "values": vb, p + "shape": np.array(shape), p + "nd": np.array(nd),
                    p + "star": np.array(star), p + "a": np.array(a), p + "b": np.array(b), p + "encoded": enc,
                    p + "recovered": sh.cpu().numpy(), p + "out_tn": out.view(torch.uint16).cpu().numpy()})
    np.savez_compressed(os.path.join(out_dir, "ref_rdp.npz"), **rdp)

    # ------------------------------------------------------------------ RS16 --
    sk = load_ref("rs_kernel16")
    from oracle.reference import init_gf_tables

    ex, lg = init_gf_tables()
    gexp = torch.from_numpy(ex).to(dev)
    glog = torch.from_numpy(lg).to(dev)
    rs = {}
    for case, (shape, k, m, miss) in enumerate([((1, 2, 12, 8), 4, 2, [0, 2]), ((1, 2, 12, 8), 8, 2, [7, 9]),
                                                ((1, 1, 10, 8), 5, 3, [1, 3, 4]), ((1, 2, 6, 8), 6, 2, [6, 1])]):
        kb = rng.standard_normal(shape).astype(np.float16).view(np.uint16)
        vb = rng.standard_normal(shape).astype(np.float16).view(np.uint16)
        N = kb.size
        kv = torch.empty(2 * N, dtype=torch.uint16, device=dev)
        sk.pack_fp16_pair_to_u16(t16(kb).reshape(-1), t16(vb).reshape(-1), kv)
        s = (2 * N + k - 1) // k
        dp = torch.zeros(k * s, dtype=torch.uint16, device=dev)
        dp[:2 * N] = kv
        sh = torch.empty((k + m, s), dtype=torch.uint16, device=dev)
        sk.encode_rs_u16(dp, sh, k, m, s, gexp, glog)
        enc = sh.cpu().numpy().copy()
        for i in miss:
            sh[i].zero_()
        md = sorted(i for i in miss if i < k)
        mp = sorted(i - k for i in miss if i >= k)
        av = [q for q in range(m) if q not in mp][:len(md)]
        sk.reconstruct_rs_u16_inplace(sh, s, k, m, torch.tensor(md, dtype=torch.int32, device=dev),
                                      torch.tensor(av, dtype=torch.int32, device=dev), gexp, glog)
        torch.cuda.synchronize()
        p = f"c{case}_"
        rs.update({p + "keys": kb, p + "values": vb, p + "shape": np.array(shape), p + "k": np.array(k),
                   p + "m": np.array(m), p + "miss": np.array(miss), p + "encoded": enc,
                   p + "recovered": sh.cpu().numpy()})
    np.savez_compressed(os.path.join(out_dir, "ref_rs16.npz"), **rs)

    # ------------------------------------------------------------ hook ext ---
    hk = load_ref("rdp_kv_ops")
    hook = {}
    for case, (world, elems, star) in enumerate([(4, 64, 0), (8, 40, 2), (2, 8, 0)]):
        ka, va = bf16_bits(rng, world * elems), bf16_bits(rng, world * elems)
        kt, vt = t16(ka), t16(va)
        S = 2 * elems
        rows = torch.empty((world + 2, S), dtype=torch.uint16, device=dev)
        for r in range(world):
            hk.pack_row_from_block(kt[r * elems:(r + 1) * elems].view(1, 1, elems, 1),
                                   vt[r * elems:(r + 1) * elems].view(1, 1, elems, 1), rows, r)
        hk.compute_rdp_parity(rows, nd=world, S=S, star_base=star)
        torch.cuda.synchronize()
        p = f"c{case}_"
        hook.update({p + "k_all": ka, p + "v_all": va, p + "world": np.array(world), p + "elems": np.array(elems),
                     p + "star": np.array(star), p + "rows": rows.cpu().numpy()})
    np.savez_compressed(os.path.join(out_dir, "ref_hook.npz"), **hook)
    print("golden vectors written to", out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
