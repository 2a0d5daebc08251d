"""Fused P2P path on real multi-GPU: one process per GPU, NCCL for control,
NVLink peer reads inside the encode kernel. Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import pytest
import torch

import mp_workers
from test_hook import run_ranks

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


@pytest.mark.parametrize("unit", [512, 4096])
def test_hook_fused_mode_two_gpus(unit):
    res = run_ranks(mp_workers.hook_fused, 2, "nccl", unit, timeout=300)
    assert res[0][1] is True
    for _rank, _ok, recs in res:
        assert recs == [1, 2, 3]


@pytest.mark.parametrize("scheme,lost_sets", [("rdp", [[1], [0], [0, 1]]), ("rs8", [[0], [1], [0, 1]]),
                                              ("xor", [[1], [0]])])
def test_hook_recover_lost_ranks_two_gpus(scheme, lost_sets):
    res = run_ranks(mp_workers.hook_recover, 2, "nccl", scheme, lost_sets, timeout=300)
    for _rank, ok, evicted in res:
        assert ok is True
        assert evicted is True


def test_hook_reads_kv_pool_through_slot_mapping_two_gpus():
    res = run_ranks(mp_workers.hook_pool, 2, "nccl", timeout=300)
    for _rank, ok, recs in res:
        assert ok is True
        assert recs == [1, 2, 3]
