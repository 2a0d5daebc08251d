"""The hook's reference-mode flow (bench_ghostserve_rdp.py:334-392, 424-476) on
the GPU against the reference's own rdp_kv_ops extension (built from its source
into oracle/_ref): ``compute_parity_to_cpu`` on world-8 gathered KV, and
``on_extend(mode="reference")`` driven through a patched FlashInfer-like
backend over NCCL (world 1 on one GPU; world 2 where two GPUs exist)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import mp_workers
from conftest import bf16_bits, pkg
from test_hook import run_ranks

pytestmark = pytest.mark.gpu


def ref_mod(name):
    build_ref = pytest.importorskip("oracle.build_ref")
    if not build_ref.built(name):
        pytest.skip(f"reference extension {name} not built")
    return build_ref.load_ref(name)


@pytest.mark.parametrize("elems,star", [(2048 * 128, 0), (2048 * 128, 5), (1000 * 3 + 1, 2)])
def test_compute_parity_to_cpu_matches_live_reference(tmp_path, rng, elems, star):
    ref = ref_mod("rdp_kv_ops")
    hook = pkg("hook")
    world = 8
    K_all = torch.from_numpy(bf16_bits(rng, world * elems)).cuda().view(torch.bfloat16)
    V_all = torch.from_numpy(bf16_bits(rng, world * elems)).cuda().view(torch.bfloat16)
    metrics = tmp_path / "ft.jsonl"
    ft = hook.KVFaultTolerance(hook.HookConfig(mode="reference", star_base=star, metrics_file=str(metrics)))
    P, Q = ft.compute_parity_to_cpu(K_all, V_all, elems, 7, 3)
    # the reference function's body, on its own extension
    S = 2 * elems
    rows = torch.empty((world + 2, S), dtype=torch.uint16, device="cuda")
    for r in range(world):
        k = K_all.narrow(0, r * elems, elems).to(torch.float16)
        v = V_all.narrow(0, r * elems, elems).to(torch.float16)
        ref.pack_row_from_block(k.view(1, 1, elems, 1), v.view(1, 1, elems, 1), rows, r)
    ref.compute_rdp_parity(rows, nd=world, S=S, star_base=star)
    torch.cuda.synchronize()
    assert P.device.type == "cpu" and Q.device.type == "cpu"
    assert torch.equal(rows[world].cpu(), P)
    assert torch.equal(rows[world + 1].cpu(), Q)
    rec = json.loads(metrics.read_text().splitlines()[-1])
    assert rec["chunk_id"] == 7 and rec["dst_rank"] == 3
    assert rec["timings"]["parity_bytes"] == 2 * S * 2
    assert set(rec["timings"]) == {"rdp_encode_ms", "rdp_decode_ms", "gpu_to_cpu_ms", "cpu_to_gpu_ms",
                                   "parity_bytes"}
    assert rec["timings"]["rdp_decode_ms"] is None
    ft.close()


@pytest.mark.parametrize("world", [1, 2])
def test_on_extend_reference_mode_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ref_mod("rdp_kv_ops")
    res = run_ranks(mp_workers.hook_reference, world, "nccl", timeout=300)
    if res[0][1] == "skip":
        pytest.skip("reference extension rdp_kv_ops not built")
    for rank, oks, recs in res:
        assert all(ok for ok, _n in oks), oks
        # the destination rank rotates with the chunk id: dst = (chunk_id - 1) % world
        assert sum(n for _ok, n in oks) == 3
        assert recs == [(cid, (cid - 1) % world) for cid in range(1, 4) if (cid - 1) % world == rank]
