"""CPU checks of the prefill harness that drives the KV hook."""
from __future__ import annotations

import pytest
import torch

from conftest import pkg

SPEC = dict(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=50)


@pytest.mark.parametrize("layout", ["pool", "layer"])
def test_chunked_prefill_equals_one_shot(layout):
    """Chunks attending to the cache prefix with lower-right causal masking give
    the same KV cache (bit for bit) and hidden states as one causal pass."""
    pre = pkg("prefill")
    spec = pre.ModelSpec(**SPEC)
    ids = torch.randint(0, 50, (48,), generator=torch.Generator().manual_seed(3))
    one = pre.TPPrefill(spec, 64, "cpu", layout=layout)
    x_all = one.forward_chunk(ids, 0)
    chunked = pre.TPPrefill(spec, 64, "cpu", layout=layout)
    outs = [chunked.forward_chunk(ids[i:i + 16], i) for i in range(0, 48, 16)]
    a, b = chunked.chunk_kv_parts(0, 48), one.chunk_kv_parts(0, 48)
    for pa, pb in zip(a[0] + a[1], b[0] + b[1]):
        assert torch.equal(pa, pb)
    assert torch.allclose(torch.cat(outs).float(), x_all.float(), atol=2e-2)


def test_layouts_compute_the_same_prefill():
    pre = pkg("prefill")
    spec = pre.ModelSpec(**SPEC)
    ids = torch.randint(0, 50, (32,), generator=torch.Generator().manual_seed(4))
    p = pre.TPPrefill(spec, 32, "cpu", layout="pool")
    q = pre.TPPrefill(spec, 32, "cpu", layout="layer")
    xp = [p.forward_chunk(ids[i:i + 8], i) for i in range(0, 32, 8)]
    xq = [q.forward_chunk(ids[i:i + 8], i) for i in range(0, 32, 8)]
    assert torch.equal(torch.cat(xp), torch.cat(xq))
    kp, vp = p.chunk_kv_parts(8, 8)
    kq, vq = q.chunk_kv_parts(8, 8)
    for a, b in zip(kp + vp, kq + vq):  # pool parts are [T, heads, D], layer-major parts [heads, T, D]
        assert torch.equal(a.transpose(0, 1), b)


def test_chunk_kv_parts_cover_the_chunk():
    pre = pkg("prefill")
    spec = pre.ModelSpec(layers=3, hidden=32, heads=2, kv_heads=1, head_dim=16, ffn=64, vocab=20)
    m = pre.TPPrefill(spec, 32, "cpu")
    m.forward_chunk(torch.arange(8) % 20, 0)
    ks, vs = m.chunk_kv_parts(0, 8)
    assert len(ks) == 3 and all(k.shape == (8, 1, 16) for k in ks)
    assert sum(k.numel() * k.element_size() for k in ks) == 3 * 8 * 16 * 2
    assert m.layer_pool(1).shape == (32, 2, 1, 16)
    assert torch.equal(m.layer_pool(1)[:8, 0], ks[1])


def test_hook_variant_calls_forward_extend_per_layer():
    """parity="hook": every layer's attention is followed by the backend's
    forward_extend with that layer's pool and the chunk's slot mapping."""
    pre = pkg("prefill")
    spec = pre.ModelSpec(layers=3, hidden=32, heads=2, kv_heads=1, head_dim=16, ffn=64, vocab=20)
    m = pre.TPPrefill(spec, 16, "cpu")
    be = pre.FlashInferAttnBackend()
    seen = []

    def forward_extend(batch, layer=None, save_kv_cache=True):
        seen.append((layer, be.kv_buffer.data_ptr(), batch.slot_mapping.tolist()))

    be.forward_extend = forward_extend
    pre.run_prefill(m, 1, 16, 8, "hook", backend=be)
    assert [s[0] for s in seen] == [0, 1, 2, 0, 1, 2]
    assert [s[1] for s in seen[:3]] == [m.layer_pool(li).data_ptr() for li in range(3)]
    assert seen[0][2] == list(range(8)) and seen[3][2] == list(range(8, 16))
