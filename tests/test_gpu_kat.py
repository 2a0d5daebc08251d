"""The CUDA encode against the committed known-answer digests
(``tests/golden/kat_codes.json``, written by ``tests/golden/kat.py`` from a
restatement of RDP and RS(k,m)/GF(2^8) that shares nothing with the oracle or
the kernels). Covers benchmark configs 0-2 at full size (32 MiB bf16 / 16 MiB
fp8 shards) and small ragged cases; the config-1 codeword is also encoded from
two-segment shards (K and V buffers) and decoded for a spread of erasure pairs.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, pkg

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import kat  # noqa: E402

pytestmark = pytest.mark.gpu

with open(kat.KAT_FILE) as _f:
    KAT = json.load(_f)["cases"]


@pytest.fixture(autouse=True)
def device_status_clean():
    yield
    assert pkg("codec").device_status(clear=True) == 0


def spec_of(rec):
    g = pkg()
    return g.CodeSpec(rec["scheme"], rec["k"], rec["m"], rec["p"], rec["unit"] or 4096)


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.cpu().numpy().view(np.uint8).tobytes()).hexdigest()


def case_tensors(case):
    return [torch.from_numpy(d).cuda() for d in kat.case_data(case)]


@pytest.mark.parametrize("case", kat.CASES, ids=[c[0] for c in kat.CASES])
def test_encode_matches_known_answer(case):
    rec = KAT[case[0]]
    g = pkg()
    par = g.encode(spec_of(rec), case_tensors(case))
    assert [t.numel() for t in par] == [rec["parity_bytes"]] * rec["m"]
    assert [digest(t) for t in par] == rec["parity_sha256"]


def test_config1_two_segment_shards_and_pairs():
    case = next(c for c in kat.CASES if c[0] == "config1_rdp_p7")
    rec = KAT[case[0]]
    g = pkg()
    spec = spec_of(rec)
    data = case_tensors(case)
    half = rec["shard_bytes"] // 2
    # each rank's shard as its K buffer and V buffer (no packing copy)
    segs = [(d[:half].clone(), d[half:].clone()) for d in data]
    par = g.encode(spec, segs)
    assert [digest(t) for t in par] == rec["parity_sha256"]
    want = [digest(d) for d in data]
    for er in ([0, 1], [2, 5], [0, 6], [3, 7], [6, 7], [4]):
        shards = list(data) + list(par)
        for e in er:
            shards[e] = None
        out = g.decode(spec, shards, er, data_bytes=rec["shard_bytes"])
        for e in er:
            got = digest(out[e])
            assert got == (want[e] if e < 6 else rec["parity_sha256"][e - 6]), (er, e)
