"""offload.HostPipeline: pinned host shards -> H2D -> encode/decode -> D2H,
checked against the device-resident engine and the CPU oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import pkg, rand_bytes
from oracle import codes

pytestmark = pytest.mark.gpu


def pinned(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


@pytest.mark.parametrize("scheme", ["rdp", "xor", "rs8"])
@pytest.mark.parametrize("nbytes,chunk", [(3 * 6 * 4096 + 4096, 6 * 4096), (1 << 20, 256 << 10), (4096, 1 << 20)])
def test_pipeline_encode_decode_match_engine(rng, scheme, nbytes, chunk):
    g, off = pkg(), pkg("offload")
    spec = {"rdp": g.CodeSpec.rdp(6, 7, 4096), "xor": g.CodeSpec.xor(6), "rs8": g.CodeSpec.rs8(6, 2)}[scheme]
    data = [rand_bytes(rng, nbytes) for _ in range(spec.k)]
    want = [t.cpu().numpy() for t in g.encode(spec, [torch.from_numpy(d).cuda() for d in data])]
    pipe = off.HostPipeline(spec, nbytes, chunk_bytes=chunk, slots=2)
    hd = [pinned(d) for d in data]
    hp = [torch.zeros(spec.parity_bytes(nbytes), dtype=torch.uint8).pin_memory() for _ in range(spec.m)]
    pipe.encode(hd, hp)
    torch.cuda.synchronize()
    for j in range(spec.m):
        assert np.array_equal(hp[j].numpy(), want[j]), j
    if scheme == "rdp":
        assert np.array_equal(hp[0].numpy(), codes.rdp_encode(data, 7, 4096)[0])
    # erase the first data shard and the last parity shard, rebuild on the host side
    er = [0, spec.k + spec.m - 1] if spec.m > 1 else [0]
    shards = hd + hp
    saved = [shards[e].clone() for e in er]
    for e in er:
        shards[e].zero_()
    pipe.decode(shards, er)
    torch.cuda.synchronize()
    for e, s in zip(er, saved):
        assert torch.equal(shards[e], s), e


def test_pipeline_overlapped_calls_then_join(rng):
    g, off = pkg(), pkg("offload")
    spec = g.CodeSpec.rdp(6, 7, 4096)
    nbytes = 40 * 6 * 4096
    pipe = off.HostPipeline(spec, nbytes, chunk_bytes=4 * 6 * 4096, slots=3)
    runs = []
    for _ in range(4):  # four different codewords in flight back to back
        data = [rand_bytes(rng, nbytes) for _ in range(spec.k)]
        hd = [pinned(d) for d in data]
        hp = [torch.empty(spec.parity_bytes(nbytes), dtype=torch.uint8).pin_memory() for _ in range(2)]
        pipe.encode(hd, hp, join=False)
        runs.append((data, hp))
    pipe.join()
    torch.cuda.current_stream().synchronize()
    for data, hp in runs:
        P, Q = codes.rdp_encode(data, 7, 4096)
        assert np.array_equal(hp[0].numpy(), P) and np.array_equal(hp[1].numpy(), Q)
