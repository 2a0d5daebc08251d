"""ctypes wrapper of the C/OpenMP oracle (oracle/cpu/liboracle.so) — TEST
INFRASTRUCTURE ONLY: the timed CPU baseline of bench.py and a second CPU check."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC_DIR = os.path.join(HERE, "cpu")
LIB_PATH = os.path.join(SRC_DIR, "liboracle.so")

_lib = None


def build() -> str:
    src = os.path.join(SRC_DIR, "oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", SRC_DIR], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        P, I, I64 = C.c_void_p, C.c_int, C.c_int64
        _lib.orc_xor_encode.argtypes = [P, I, I64, P, I]
        _lib.orc_rdp_encode.argtypes = [P, I, I, I64, I64, P, P, I]
        _lib.orc_rs8_encode.argtypes = [P, I, I, I64, P, I]
        _lib.orc_rs16_encode.argtypes = [P, I, I, I64, P, I]
        _lib.orc_rdpref_parity.argtypes = [P, I, I64, I, I]
        _lib.orc_max_threads.restype = I
    return _lib


def _ptrs(arrs):
    return (C.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])


def max_threads() -> int:
    return int(lib().orc_max_threads())


def xor_encode(data, threads=0) -> np.ndarray:
    out = np.empty_like(data[0])
    lib().orc_xor_encode(_ptrs(data), len(data), data[0].size, out.ctypes.data, threads)
    return out


def rdp_encode(data, p, unit, threads=0, out=None):
    sb = (p - 1) * unit
    nb = -(-data[0].size // sb) * sb
    if out is None:
        out = (np.empty(nb, np.uint8), np.empty(nb, np.uint8))
    lib().orc_rdp_encode(_ptrs(data), len(data), p, unit, data[0].size, out[0].ctypes.data, out[1].ctypes.data,
                         threads)
    return out


def rs8_encode(data, m, threads=0, out=None):
    if out is None:
        out = [np.empty_like(data[0]) for _ in range(m)]
    lib().orc_rs8_encode(_ptrs(data), len(data), m, data[0].size, _ptrs(out), threads)
    return out


def rs16_encode(data_padded: np.ndarray, k: int, m: int, s: int, threads=0) -> np.ndarray:
    out = np.empty(m * s, np.uint16)
    lib().orc_rs16_encode(data_padded.ctypes.data, k, m, s, out.ctypes.data, threads)
    return out.reshape(m, s)


def rdpref_parity(rows: np.ndarray, nd: int, S: int, star_base: int, threads=0) -> np.ndarray:
    rows = np.ascontiguousarray(rows)
    lib().orc_rdpref_parity(rows.ctypes.data, nd, S, star_base, threads)
    return rows
