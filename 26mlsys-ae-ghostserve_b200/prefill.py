"""Tensor-parallel chunked prefill that drives the KV hook — the harness for
measuring what parity costs a prefill (prefill tokens/s with vs without it).

The reference measures this inside an SGLang server (bench_ghostserve_rdp.py:
544-704: TP=8, chunked prefill, FlashInfer attention, TTFT over HTTP).  SGLang
is not part of this project; this module is the smallest prefill that produces
the same KV traffic: a Llama-3.1-8B-architecture decoder (32 layers, hidden
4096, 32 query / 8 KV heads of 128, FFN 14336, vocab 128256, RoPE theta 5e5,
random bf16 weights) split Megatron-style over the ranks of a process group:

* QKV and gate/up projections column-parallel, O and down projections
  row-parallel followed by an all-reduce (NCCL);
* every rank owns kv_heads / world KV heads of the KV cache (layouts below);
* a chunk of T tokens at position p attends to the cache prefix [0, p + T) with
  lower-right causal masking (scaled_dot_product_attention, grouped-query).

KV cache layout: SGLang's FlashInfer pool, one pool per layer of
``[max_tokens, 2 (K, V), kv_heads_rank, 128]`` (``layout="pool"``, the
default; slot = token position), or a layer-major ``[layers, kv_heads_rank,
max_tokens, 128]`` pair (``layout="layer"``).

Parity variants (``run_prefill``):
* ``"hook"``: the drop-in hook as SGLang drives it — a FlashInfer-named
  attention backend patched with ``hook.patch_backend``; after every layer's
  attention its ``forward_extend`` is called with the chunk's slot mapping and
  that layer's pool, so the hook (``protect="call"``) encodes every layer's
  delta KV separately, 32 times per chunk, like the reference hook
  (bench_ghostserve_rdp.py:424-476);
* ``"hook_chunk"``: the same calls with ``protect="chunk"``: the hook keeps the
  layers' pools and encodes once per chunk, after the last layer's call (one
  gather launch over all layers, one barrier, one sliced encode, one host copy);
* ``"fused"``: after all layers of a chunk, ``KVFaultTolerance.encode_parts``
  on the chunk's K and V views of every layer (staged by copies);
* ``"reference"``: the reference hook's flow after every layer's attention
  (chunk id broadcast, gather to the rotating destination, fp16 cast, mod-S
  parity, synchronous copy to the host), once per forward_extend call.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch.nn.attention.bias import causal_lower_right


@dataclass(frozen=True)
class ModelSpec:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    eps: float = 1e-5


class TPPrefill:
    """One rank's slice of the model and its KV cache."""

    def __init__(self, spec: ModelSpec, max_tokens: int, device, group=None, seed: int = 0, layout: str = "pool"):
        self.spec = spec
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        w = self.world
        if spec.heads % w or spec.kv_heads % w or spec.ffn % w:
            raise ValueError(f"world {w} must divide heads, kv_heads and ffn")
        self.hq, self.hk, self.f = spec.heads // w, spec.kv_heads // w, spec.ffn // w
        self.device = torch.device(device)
        D, H = spec.head_dim, spec.hidden
        gen = torch.Generator(device=self.device).manual_seed(seed * 1000 + self.rank)

        def rnd(*shape, std=0.02):
            return (torch.randn(*shape, generator=gen, device=self.device, dtype=torch.bfloat16) * std)

        self.layers = []
        for _ in range(spec.layers):
            self.layers.append(dict(
                wqkv=rnd(H, (self.hq + 2 * self.hk) * D), wo=rnd(self.hq * D, H),
                w13=rnd(H, 2 * self.f), w2=rnd(self.f, H),
                ln1=torch.ones(H, device=self.device, dtype=torch.bfloat16),
                ln2=torch.ones(H, device=self.device, dtype=torch.bfloat16)))
        self.embed = rnd(spec.vocab, H, std=1.0)
        if layout not in ("pool", "layer"):
            raise ValueError("layout must be 'pool' or 'layer'")
        self.layout = layout
        if layout == "pool":  # per layer [slots, 2, kv_heads, D]: slot s holds token s's K and V
            self.pool = torch.empty(spec.layers, max_tokens, 2, self.hk, D, device=self.device, dtype=torch.bfloat16)
        else:
            self.kcache = torch.empty(spec.layers, self.hk, max_tokens, D, device=self.device, dtype=torch.bfloat16)
            self.vcache = torch.empty_like(self.kcache)
        inv = 1.0 / (spec.rope_theta ** (torch.arange(0, D, 2, device=self.device, dtype=torch.float32) / D))
        ang = torch.outer(torch.arange(max_tokens, device=self.device, dtype=torch.float32), inv)
        self.cos, self.sin = ang.cos(), ang.sin()
        self.max_tokens = max_tokens

    def _norm(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.spec.eps)).to(x.dtype) * w

    def _rope(self, x, pos0):
        """Rotate-half RoPE on [T, heads, D]."""
        T = x.shape[0]
        c = self.cos[pos0:pos0 + T, None, :]
        s = self.sin[pos0:pos0 + T, None, :]
        x1, x2 = x.float().chunk(2, dim=-1)
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)

    def _all_reduce(self, t):
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def forward_chunk(self, ids: torch.Tensor, pos0: int,
                      after_attention: Optional[Callable[[int, torch.Tensor, torch.Tensor], None]] = None):
        """Run one chunk through every layer, writing its K/V into the cache."""
        T = ids.numel()
        if pos0 + T > self.max_tokens:
            raise ValueError("chunk past the end of the KV cache")
        D, hq, hk = self.spec.head_dim, self.hq, self.hk
        x = self.embed[ids]
        mask = causal_lower_right(T, pos0 + T)
        for li, L in enumerate(self.layers):
            h = self._norm(x, L["ln1"])
            qkv = h @ L["wqkv"]
            q = self._rope(qkv[:, :hq * D].view(T, hq, D), pos0)
            k = self._rope(qkv[:, hq * D:(hq + hk) * D].view(T, hk, D), pos0)
            v = qkv[:, (hq + hk) * D:].view(T, hk, D)
            if self.layout == "pool":
                self.pool[li, pos0:pos0 + T, 0] = k
                self.pool[li, pos0:pos0 + T, 1] = v
                kc = self.pool[li, :pos0 + T, 0].transpose(0, 1)
                vc = self.pool[li, :pos0 + T, 1].transpose(0, 1)
            else:
                self.kcache[li, :, pos0:pos0 + T] = k.transpose(0, 1)
                self.vcache[li, :, pos0:pos0 + T] = v.transpose(0, 1)
                kc, vc = self.kcache[li, :, :pos0 + T], self.vcache[li, :, :pos0 + T]
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], kc[None], vc[None], attn_mask=mask,
                                               enable_gqa=hq != hk)
            if after_attention is not None:
                after_attention(li, kc[:, pos0:pos0 + T], vc[:, pos0:pos0 + T])
            o = o[0].transpose(0, 1).reshape(T, hq * D) @ L["wo"]
            x = x + self._all_reduce(o)
            h = self._norm(x, L["ln2"])
            gu = h @ L["w13"]
            a = F.silu(gu[:, :self.f]) * gu[:, self.f:]
            x = x + self._all_reduce(a @ L["w2"])
        return x

    def chunk_kv_parts(self, pos0: int, T: int):
        """The chunk's K and V of every layer on this rank (views into the cache)."""
        if self.layout == "pool":
            return ([self.pool[li, pos0:pos0 + T, 0] for li in range(self.spec.layers)],
                    [self.pool[li, pos0:pos0 + T, 1] for li in range(self.spec.layers)])
        return ([self.kcache[li, :, pos0:pos0 + T] for li in range(self.spec.layers)],
                [self.vcache[li, :, pos0:pos0 + T] for li in range(self.spec.layers)])

    def layer_pool(self, li: int) -> torch.Tensor:
        """Layer li's KV pool [slots, 2, kv_heads_rank, head_dim] (layout "pool")."""
        return self.pool[li]


class FlashInferAttnBackend:
    """The attention-backend object the hook patches (it only needs the class
    name, ``forward_extend`` and the pool attribute). ``kv_buffer`` is set to
    the pool of the layer whose extend call is being made."""

    def __init__(self):
        self.kv_buffer = None

    def forward_extend(self, batch, layer=None, save_kv_cache=True):
        return None


class ExtendBatch:
    """The part of SGLang's forward batch the hook reads: the chunk's slot mapping."""

    def __init__(self, slot_mapping: torch.Tensor):
        self.slot_mapping = slot_mapping


def run_prefill(model: TPPrefill, seqs: int, seq_len: int, chunk: int, parity: str, ft=None, seed: int = 1,
                backend: Optional[FlashInferAttnBackend] = None) -> int:
    """Prefill `seqs` sequences of `seq_len` random token ids chunk by chunk;
    returns the number of tokens processed. parity "hook"/"hook_chunk" need
    `backend`, a FlashInferAttnBackend patched with hook.patch_backend(backend, ft)."""
    gen = torch.Generator(device=model.device).manual_seed(seed)
    cid = 0
    for _ in range(seqs):
        ids = torch.randint(0, model.spec.vocab, (seq_len,), generator=gen, device=model.device)
        for pos0 in range(0, seq_len, chunk):
            T = min(chunk, seq_len - pos0)
            cb = None
            if parity == "reference":
                def cb(li, k, v):  # the reference hook, once per layer's extend call
                    chunk_id, dst = ft.next_chunk_id(device=model.device)
                    got = ft.gather_kv(k.transpose(0, 1), v.transpose(0, 1), dst)
                    if got is not None:
                        ft.compute_parity_to_cpu(*got, chunk_id, dst)
            elif parity in ("hook", "hook_chunk"):
                batch = ExtendBatch(torch.arange(pos0, pos0 + T, device=model.device, dtype=torch.int64))

                def cb(li, k, v, batch=batch):  # SGLang's extend call of layer li
                    backend.kv_buffer = model.layer_pool(li)
                    backend.forward_extend(batch, layer=li)
            model.forward_chunk(ids[pos0:pos0 + T], pos0, after_attention=cb)
            if parity == "fused":
                cid += 1
                ks, vs = model.chunk_kv_parts(pos0, T)
                ft.encode_parts(ks, vs, cid)
    return seqs * seq_len
