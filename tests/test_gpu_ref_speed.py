"""The engine's drop-ins against the reference's own CUDA kernels on the same
bytes: every pair agrees bit for bit. Speed is reported by bench.py
(``--workload refcompat``), not asserted here."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_dropins_match_reference_kernels():
    pytest.importorskip("oracle.build_ref")
    import ref_speed

    res = ref_speed.measure(T=1024, n=2048, reps=10)
    pairs = {k: v for k, v in res.items() if isinstance(v, dict)}
    if not pairs:
        pytest.skip("no reference extension built")
    for name, r in pairs.items():
        assert r["equal"], name
