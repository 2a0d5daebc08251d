"""ctypes binding of libgsec.so (the C ABI declared in include/gsec.h).

The library is loaded from ``lib/libgsec.so`` next to this file.  There is no
fallback: if the library is missing, or a call is made without a CUDA device,
the call raises.  Return codes map to exceptions the way the reference's own
errors do (``ValueError`` for bad arguments, ``RuntimeError`` otherwise).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libgsec.so")

GSEC_OK = 0
GSEC_EINVAL = 1
GSEC_EUNRECOVERABLE = 2
GSEC_ECUDA = 3
GSEC_ETIMEOUT = 4
GSEC_EUNSUPPORTED = 5

SCHEME_XOR = 0
SCHEME_RDP = 1
SCHEME_RS8 = 2

IPC_HANDLE_BYTES = 64


class GsecError(RuntimeError):
    """A libgsec call failed (CUDA error, timeout, unsupported parameters)."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class GsecArgumentError(GsecError, ValueError):
    """A libgsec call rejected its arguments (GSEC_EINVAL)."""


class GsecUnrecoverable(GsecError):
    """The erasure pattern cannot be decoded (GSEC_EUNRECOVERABLE)."""


class Code(C.Structure):
    """struct gsec_code."""
    _fields_ = [("scheme", C.c_int32), ("k", C.c_int32), ("m", C.c_int32), ("p", C.c_int32),
                ("unit", C.c_int64)]


_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_PP = C.POINTER(C.c_void_p)
_PI32 = C.POINTER(C.c_int32)

_SIGS = {
    "gsec_last_error": (C.c_char_p, []),
    "gsec_version": (C.c_char_p, []),
    "gsec_device_status": (C.c_int, [C.POINTER(C.c_uint32), _I32]),
    "gsec_parity_bytes": (C.c_int, [C.POINTER(Code), _I64, C.POINTER(_I64)]),
    "gsec_encode": (C.c_int, [C.POINTER(Code), _PP, _PP, _I64, _I64, _PP, _I64, _I64, _P]),
    "gsec_decode": (C.c_int, [C.POINTER(Code), _PP, _PP, _I64, _I64, _PI32, _I32, _I64, _I64, _P]),
    "gsec_rows_pack": (C.c_int, [_P, _I64, _P, _I64, _P, _I64, _I64, _I32, _P]),
    "gsec_rows_unpack": (C.c_int, [_P, _I64, _I64, _I32, _P, _I64, _P, _I64, _P]),
    "gsec_copy_async": (C.c_int, [_P, _P, _I64, _P]),
    "gsec_copy_gather": (C.c_int, [_PP, C.POINTER(_I64), _I32, _P, _P]),
    "gsec_slots_gather": (C.c_int, [_P, _I64, _I64, _I32, _I64, _P, _I32, _I64, _I64, _P, _P]),
    "gsec_slots_scatter": (C.c_int, [_P, _I64, _I64, _I32, _I64, _P, _I32, _I64, _I64, _P, _P]),
    "gsec_slots_gather_pools": (C.c_int, [_PP, _I32, _I64, _I64, _I32, _I64, _P, _I32, _I64, _I64, _P, _P, _I64,
                                          _P]),
    "gsec_slots_scatter_pools": (C.c_int, [_PP, _I32, _I64, _I64, _I32, _I64, _P, _I32, _I64, _I64, _P, _P, _I64,
                                           _P]),
    "gsec_xor_encode": (C.c_int, [_P, _P, _I32, _I64, _I64, _P]),
    "gsec_xor_reconstruct": (C.c_int, [_P, _P, _I64, _I64, _I32, _PI32, _I32, _P]),
    "gsec_rdpref_pack_row": (C.c_int, [_P, _P, _I64, _P, _I64, _I32, _P]),
    "gsec_rdpref_parity": (C.c_int, [_P, _I64, _I32, _I64, _I32, _P]),
    "gsec_rdpref_backup": (C.c_int, [_P, _P, _P, _I64, _I32, _I64, _I64, _I64, _I32, _P]),
    "gsec_rdpref_backup_bhtd": (C.c_int, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, _I32, _I64, _I32, _P]),
    "gsec_rdpref_recovery": (C.c_int, [_P, _I64, _P, _I32, _I64, _I64, _I64, _I32, _I32, _I32, _P]),
    "gsec_rdpref_recovery_bhtd": (C.c_int, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I32, _I64, _I32, _I32,
                                            _I32, _P]),
    "gsec_rs16_tables": (C.c_int, [_P, _P]),
    "gsec_rs16_encode": (C.c_int, [_P, _P, _I64, _I32, _I32, _I64, _P]),
    "gsec_rs16_reconstruct": (C.c_int, [_P, _I64, _I64, _I32, _I32, _PI32, _I32, _PI32, _P]),
    "gsec_ipc_export": (C.c_int, [_P, _P, C.POINTER(_I64)]),
    "gsec_ipc_import": (C.c_int, [_P, _I64, C.POINTER(C.c_void_p)]),
    "gsec_ipc_close_all": (C.c_int, []),
}

_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Load libgsec.so once; raise if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"libgsec.so not built at {LIB_PATH}; run 26mlsys-ae-ghostserve_b200/build.py")
                h = C.CDLL(LIB_PATH)
                for name, (res, args) in _SIGS.items():
                    fn = getattr(h, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = h
    return _lib


def exported_names():
    return list(_SIGS)


def check(rc: int) -> None:
    if rc == GSEC_OK:
        return
    msg = lib().gsec_last_error().decode(errors="replace")
    if rc == GSEC_EINVAL:
        raise GsecArgumentError(rc, msg)
    if rc == GSEC_EUNRECOVERABLE:
        raise GsecUnrecoverable(rc, msg)
    raise GsecError(rc, msg)


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def ptr_array(ptrs) -> C.Array:
    return (C.c_void_p * max(1, len(ptrs)))(*[C.c_void_p(int(p)) if p else None for p in ptrs])


def i32_array(vals) -> C.Array:
    return (C.c_int32 * max(1, len(vals)))(*[int(v) for v in vals])
