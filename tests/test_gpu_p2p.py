"""Multi-process path on one GPU: two ranks share KV through CUDA IPC and each
encodes its stripe slice by reading the other's memory through mapped pointers
(the kernel path used over NVLink on several GPUs). gloo carries control only;
nothing waits on a device flag."""
from __future__ import annotations

import pytest

import mp_workers
from test_hook import run_ranks

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scheme", ["rdp", "xor", "rs8"])
def test_ipc_sliced_encode_two_ranks(scheme):
    res = run_ranks(mp_workers.ipc_sliced_encode, 2, scheme, timeout=300)
    assert res[0][1] is True


@pytest.mark.parametrize("unit", [512, 4096])
def test_hook_fused_mode_two_ranks(unit):
    res = run_ranks(mp_workers.hook_fused, 2, "gloo", unit, timeout=300)
    assert res[0][1] is True
    for _rank, _ok, recs in res:
        assert recs == [1, 2, 3]


@pytest.mark.parametrize("scheme,lost_sets", [("rdp", [[1], [0], [0, 1]]), ("rs8", [[0], [1], [0, 1]]),
                                              ("xor", [[1], [0]])])
def test_hook_recover_lost_ranks(scheme, lost_sets):
    res = run_ranks(mp_workers.hook_recover, 2, "gloo", scheme, lost_sets, timeout=300)
    for _rank, ok, evicted in res:
        assert ok is True
        assert evicted is True


def test_hook_reads_kv_pool_through_slot_mapping():
    res = run_ranks(mp_workers.hook_pool, 2, "gloo", timeout=300)
    for _rank, ok, recs in res:
        assert ok is True
        assert recs == [1, 2, 3]


def test_hook_chunk_mode_encodes_all_layers_once():
    res = run_ranks(mp_workers.hook_pool_chunk, 2, "gloo", timeout=300)
    for _rank, ok, recs in res:
        assert ok is True
        assert recs == [1, 2]
