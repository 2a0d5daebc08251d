"""gsec — B200-native erasure coding for tensor-parallel KV caches.

Host layer (Python/PyTorch) over libgsec.so, a C-ABI library of hand-written
sm_100a kernels.  Import with ``importlib.import_module("26mlsys-ae-ghostserve_b200")``
(the directory name is not a Python identifier).

Submodules
----------
codec       engine encode/decode (XOR, textbook RDP, RS over GF(2^8)) on shards in
            GPU memory, including peer-mapped shards of other ranks
ext         the reference's extension-level function names (xor_kernel, rdp_kernel,
            rs_kernel, rdp_kv_ops)
benchmark   drop-ins for the reference's benchmark/{xor,rdp,rs}/main.py
hook        drop-in for the reference's SGLang forward_extend KV hook
p2p         CUDA-IPC peer mapping of KV buffers across the ranks of a node
offload     pinned-host parity ring: pipelined device<->host encode and restore
"""
from . import _lib  # noqa: F401
from .codec import CodeSpec, decode, encode, parity_bytes  # noqa: F401

__all__ = ["CodeSpec", "encode", "decode", "parity_bytes"]
