"""CPU checks of the prefill harness that drives the KV hook."""
from __future__ import annotations

import torch

from conftest import pkg


def test_chunked_prefill_equals_one_shot():
    """Chunks attending to the cache prefix with lower-right causal masking give
    the same KV cache (bit for bit) and hidden states as one causal pass."""
    pre = pkg("prefill")
    spec = pre.ModelSpec(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, ffn=96, vocab=50)
    ids = torch.randint(0, 50, (48,), generator=torch.Generator().manual_seed(3))
    one = pre.TPPrefill(spec, 64, "cpu")
    x_all = one.forward_chunk(ids, 0)
    chunked = pre.TPPrefill(spec, 64, "cpu")
    outs = [chunked.forward_chunk(ids[i:i + 16], i) for i in range(0, 48, 16)]
    assert torch.equal(chunked.kcache[:, :, :48], one.kcache[:, :, :48])
    assert torch.equal(chunked.vcache[:, :, :48], one.vcache[:, :, :48])
    assert torch.allclose(torch.cat(outs).float(), x_all.float(), atol=2e-2)


def test_chunk_kv_parts_cover_the_chunk():
    pre = pkg("prefill")
    spec = pre.ModelSpec(layers=3, hidden=32, heads=2, kv_heads=1, head_dim=16, ffn=64, vocab=20)
    m = pre.TPPrefill(spec, 32, "cpu")
    m.forward_chunk(torch.arange(8) % 20, 0)
    ks, vs = m.chunk_kv_parts(0, 8)
    assert len(ks) == 3 and all(k.shape == (1, 8, 16) for k in ks)
    assert sum(k.numel() * k.element_size() for k in ks) == 3 * 8 * 16 * 2
