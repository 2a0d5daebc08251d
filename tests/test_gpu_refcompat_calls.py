"""The reference-layout calls bench.py times (``--workload refcompat``), run
through both arms in one process on the same bytes: this package's drop-ins
and the reference's own CUDA extensions (built from its sources into
oracle/_ref) must give identical outputs for every call. Speed is reported by
bench.py, not asserted here."""
from __future__ import annotations

import importlib.util
import os

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def bench_module():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("T,n", [(1024, 2048), (257, 1280)])
def test_refcompat_calls_match_reference_kernels(T, n):
    pytest.importorskip("oracle.build_ref")
    bench = bench_module()
    ref = bench.refcompat_calls("reference", T, n)
    if ref is None:
        pytest.skip("reference extensions not built")
    ours = bench.refcompat_calls("ours", T, n)
    assert sorted(ref) == sorted(ours)
    for name in ref:
        for calls in (ref, ours):
            calls[name][0]()
        torch.cuda.synchronize()
        a, b = ref[name][1](), ours[name][1]()
        assert a.shape == b.shape, name
        assert torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8)), name
