"""Host-side behaviour of the KV hook drop-in (CPU; gloo ranks for collectives)."""
from __future__ import annotations

import json
import socket

import pytest
import torch
import torch.multiprocessing as mp

import mp_workers
from conftest import pkg


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def run_ranks(fn, world, *args, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    try:
        import queue as _queue
        import time as _time
        deadline = _time.monotonic() + timeout
        while len(res) < len(procs):
            try:
                res.append(q.get(timeout=1.0))
            except _queue.Empty:
                # a rank that died leaves the others waiting on it: fail now
                dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
                assert not dead, f"a rank exited with {dead}"
                assert _time.monotonic() < deadline, "ranks timed out"
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return sorted(res, key=lambda r: r[0])


class FakeFlashInferAttnBackend:
    def __init__(self):
        self.kv_pool = torch.zeros(8, 2, 1, 4)
        self.calls = 0

    def forward_extend(self, batch, layer=None, save_kv_cache=True):
        self.calls += 1
        return ("out", batch, layer, save_kv_cache)


class RaisingFT:
    def __init__(self):
        self.seen = 0

    def on_extend(self, batch, kv_pool):
        self.seen += 1
        raise RuntimeError("boom")


def test_patch_forwards_arguments_and_swallows_errors(capsys):
    hook = pkg("hook")
    be = FakeFlashInferAttnBackend()
    ft = RaisingFT()
    assert hook.patch_backend(be, ft)
    assert hook.patch_backend(be, ft)  # idempotent
    res = be.forward_extend("batch", layer=3, save_kv_cache=False)
    assert res == ("out", "batch", 3, False)
    assert be.calls == 1 and ft.seen == 1
    assert "FlashInfer hook error: boom" in capsys.readouterr().out


def test_patch_skips_other_backends():
    hook = pkg("hook")

    class TritonBackend:
        def forward_extend(self, *a):
            return 1

    assert not hook.patch_backend(TritonBackend(), RaisingFT())


def test_patch_model_runner():
    hook = pkg("hook")

    class MR:
        attn_backend = FakeFlashInferAttnBackend()

    assert hook.patch_model_runner(MR(), RaisingFT())


def test_on_extend_without_process_group_is_a_no_op():
    hook = pkg("hook")
    ft = hook.KVFaultTolerance(hook.HookConfig(metrics_file=None))

    class Batch:
        slot_mapping = torch.tensor([0, 1, -1])

    ft.on_extend(Batch(), torch.zeros(4, 2, 1, 8))  # no process group: returns like the reference
    assert ft.records == []


def test_metrics_record_schema(tmp_path):
    hook = pkg("hook")
    f = tmp_path / "m.jsonl"
    ft = hook.KVFaultTolerance(hook.HookConfig(metrics_file=str(f)))
    rec = ft._record(3, 2, 0.5, 0.25, 0.125, 1024)
    ft._emit(rec)
    line = json.loads(f.read_text().strip())
    assert set(line) == {"chunk_id", "dst_rank", "first_chunk_wall_ms", "timings"}
    assert set(line["timings"]) == {"rdp_encode_ms", "rdp_decode_ms", "gpu_to_cpu_ms", "cpu_to_gpu_ms",
                                    "parity_bytes"}
    assert line["chunk_id"] == 3 and line["timings"]["rdp_decode_ms"] is None


@pytest.mark.parametrize("mode", ["reference", "fused"])
def test_chunk_ids_rotate_destination(mode):
    res = run_ranks(mp_workers.chunk_ids, 2, mode)
    for _rank, ids in res:
        assert ids == [(c, (c - 1) % 2) for c in range(1, 6)]


def test_reference_gather_to_rotating_destination():
    res = run_ranks(mp_workers.gather, 3)
    assert [r[1] for r in res] == [0, 1, 2]
    for _rank, _dst, elems, k_all, v_all in res:
        assert elems == 12
        assert k_all == [float(r) for r in range(3) for _ in range(12)]
        assert v_all == [float(10 + r) for r in range(3) for _ in range(12)]


def test_peer_table_exchange():
    res = run_ranks(mp_workers.peer_table, 2)
    for rank, table in res:
        other = 1 - rank
        assert table[other] == [1000 * other + 16 * (j + 1) for j in range(3)]
        assert len(table[rank]) == 3


def test_stripe_slices_partition():
    p2p = pkg("p2p")
    for n in (0, 1, 7, 8, 1366):
        for w in (1, 2, 3, 8):
            cuts = [p2p.stripe_slice(r, w, n) for r in range(w)]
            assert cuts[0][0] == 0 and cuts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(cuts, cuts[1:]))
            sizes = [b - a for a, b in cuts]
            assert max(sizes) - min(sizes) <= 1
    assert p2p.codeword_placement(3, 8, 6) == [3, 4, 5, 6, 7, 0]


def test_chunk_mode_encodes_once_per_chunk():
    res = run_ranks(mp_workers.chunk_mode_calls, 1)
    _rank, got = res[0]
    assert [g[0] for g in got] == [[0, 1, 2], [0, 1, 2]]  # the chunk's pools, in layer order
    assert [g[1] for g in got] == [1, 2]                  # one chunk id per chunk
    assert got[1][2] == [4, 5, 6, 7]
