"""CPU checks of the C-ABI library: it loads, exports every symbol the header
declares, and rejects bad arguments before touching a GPU."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, pkg
from oracle import reference as R

HEADER = os.path.join(ROOT, "include", "gsec.h")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"GSEC_API\s+(?:const\s+)?\w+\*?\s+(gsec_\w+)\(", txt)))


def test_header_declares_the_abi():
    syms = header_symbols()
    assert len(syms) >= 20
    assert {"gsec_encode", "gsec_decode", "gsec_rdpref_parity", "gsec_rs16_reconstruct"} <= set(syms)


def test_library_exports_every_declared_symbol():
    lib = pkg("_lib").lib()
    for name in header_symbols():
        assert hasattr(lib, name), name
    assert set(pkg("_lib").exported_names()) == set(header_symbols())


def test_version_and_no_error():
    lib = pkg("_lib").lib()
    assert lib.gsec_version().startswith(b"gsec ")


def test_parity_bytes():
    g = pkg()
    assert g.parity_bytes(g.CodeSpec.rdp(6, 7), 32 << 20) == 1366 * 6 * 4096
    assert g.parity_bytes(g.CodeSpec.rdp(6, 7, unit=16), 96) == 96
    assert g.parity_bytes(g.CodeSpec.rs8(6, 2), 16 << 20) == 16 << 20
    for k in range(1, 17):
        spec = g.CodeSpec.rdp(k)
        assert spec.p - 1 >= k
        assert g.parity_bytes(spec, 12345 * 16) == spec.parity_bytes(12345 * 16)


@pytest.mark.parametrize("spec_args,err", [
    (("rdp", 7, 2, 7, 4096), "k=7"),
    (("rdp", 4, 2, 9, 4096), "p=9"),
    (("rdp", 4, 2, 5, 24), "unit"),
    (("xor", 3, 2, 0, 0), "m=2"),
    (("rs8", 6, 5, 0, 0), "m=5"),
    (("rs8", 0, 2, 0, 0), "k=0"),
])
def test_bad_code_parameters(spec_args, err):
    g = pkg()
    with pytest.raises((ValueError, RuntimeError), match=err):
        g.parity_bytes(g.CodeSpec(*spec_args), 4096)


def _code(spec):
    return spec.c_code()


def test_encode_argument_checks_run_on_host():
    g = pkg()
    L = pkg("_lib")
    spec = g.CodeSpec.rdp(6, 7)
    code = _code(spec)
    fake = [0x10000 * (i + 1) for i in range(6)]
    par = [0x900000, 0xA00000]
    # data_bytes not a multiple of 16
    with pytest.raises(ValueError, match="multiple of 16"):
        L.call("gsec_encode", ctypes.byref(code), L.ptr_array(fake), None, 0, 100, L.ptr_array(par), 0, 24576, None)
    # misaligned data pointer
    bad = list(fake)
    bad[2] += 8
    with pytest.raises(ValueError, match="aligned"):
        L.call("gsec_encode", ctypes.byref(code), L.ptr_array(bad), None, 0, 4096, L.ptr_array(par), 0, 24576, None)
    # range not stripe aligned
    with pytest.raises(ValueError, match="aligned"):
        L.call("gsec_encode", ctypes.byref(code), L.ptr_array(fake), None, 0, 49152, L.ptr_array(par), 16, 24576,
               None)


def test_decode_rejects_too_many_erasures_on_host():
    g = pkg()
    L = pkg("_lib")
    spec = g.CodeSpec.rdp(6, 7)
    code = _code(spec)
    ptrs = [0x10000 * (i + 1) for i in range(8)]
    with pytest.raises(L.GsecUnrecoverable):
        L.call("gsec_decode", ctypes.byref(code), L.ptr_array(ptrs), None, 0, 4096, L.i32_array([0, 1, 2]), 3, 0,
               24576, None)
    with pytest.raises(ValueError, match="repeated"):
        L.call("gsec_decode", ctypes.byref(code), L.ptr_array(ptrs), None, 0, 4096, L.i32_array([1, 1]), 2, 0,
               24576, None)


def test_rs16_tables_match_reference_restatement():
    rs = pkg("benchmark.rs.main")
    ex, lg = rs.init_gf_tables()
    ex2, lg2 = R.init_gf_tables()
    assert np.array_equal(ex, ex2) and np.array_equal(lg, lg2)


def test_dropins_reject_cpu_tensors_like_the_reference():
    x = torch.zeros(1, 2, 4, 8, dtype=torch.float16)
    with pytest.raises(AssertionError):
        pkg("benchmark.xor.main").forward_encode_kv(x, x, 4, 1)
    with pytest.raises(ValueError):
        pkg("benchmark.xor.main").forward_encode_kv(x, x, 4, 2)
    with pytest.raises(ValueError, match="CUDA"):
        pkg("benchmark.rdp.main").fused_backup_full_kv(x, x, 4)
    with pytest.raises(AssertionError):
        pkg("benchmark.rs.main").forward_encode_kv(x, x, 4, 2)
    with pytest.raises(ValueError):
        pkg("benchmark.rdp.main").determine_shard_size_words(10, 0)


def test_shard_size_helpers_match_reference():
    x = pkg("benchmark.xor.main")
    r = pkg("benchmark.rdp.main")
    s = pkg("benchmark.rs.main")
    for total in (1, 7, 100, 4096, 12345):
        for k in (1, 3, 6, 7, 8):
            assert x.determine_shard_size(total, k) == R.determine_shard_size(total, k)
            assert r.determine_shard_size_words(total, k) == R.determine_shard_size_words(total, k)
            assert s.shard_size_and_pad(total, k) == R.shard_size_and_pad(total, k)


def test_engine_requires_cuda_tensors():
    g = pkg()
    with pytest.raises(ValueError, match="CUDA"):
        g.encode(g.CodeSpec.xor(2), [torch.zeros(32, dtype=torch.uint8)] * 2)


def test_slot_and_copy_argument_checks_run_on_host():
    """Calls that fail on the first null-pointer or size check, before any later
    check could let them reach a launch: the fake addresses are never used."""
    L = pkg("_lib")
    P = ctypes.c_void_p
    # slot list element size
    with pytest.raises(ValueError, match="slot_bytes"):
        L.call("gsec_slots_gather", P(0x10000), 512, 256, 1, 256, P(0x20000), 3, 4, 64, P(0x30000), None)
    # null pool / destination
    with pytest.raises(ValueError, match="null"):
        L.call("gsec_slots_gather", None, 512, 256, 1, 256, P(0x20000), 8, 4, 64, P(0x30000), None)
    with pytest.raises(ValueError, match="null"):
        L.call("gsec_slots_scatter", P(0x10000), 512, 256, 1, 256, P(0x20000), 8, 4, 64, None, None)
    with pytest.raises(ValueError):
        L.call("gsec_copy_async", P(0x10000), P(0x20000), -1, None)
    with pytest.raises(ValueError, match="null"):
        L.call("gsec_copy_async", None, P(0x20000), 16, None)
    L.call("gsec_copy_async", None, None, 0, None)  # nothing to copy


@pytest.mark.skipif(torch.cuda.is_available(), reason="fake device addresses: host-only machine")
def test_slot_record_checks_run_on_host():
    """Alignment, record geometry and the empty list: checks that come after
    the null/size checks. With a GPU present a loosened check could launch on
    the fake addresses, so these run only where no GPU exists."""
    L = pkg("_lib")
    P = ctypes.c_void_p
    # rows that are not whole 16-byte vectors
    with pytest.raises(ValueError, match="16-byte"):
        L.call("gsec_slots_gather", P(0x10000), 512, 256, 1, 200, P(0x20000), 8, 4, 64, P(0x30000), None)
    # planes that do not fit in the slot record, negative plane offset, zero pitch
    for fn in ("gsec_slots_gather", "gsec_slots_scatter"):
        with pytest.raises(ValueError, match="slot record"):
            L.call(fn, P(0x10000), 512, 256, 2, 512, P(0x20000), 8, 4, 64, P(0x30000), None)
        with pytest.raises(ValueError, match="slot record"):
            L.call(fn, P(0x10000), 512, -256, 2, 256, P(0x20000), 8, 4, 64, P(0x30000), None)
        with pytest.raises(ValueError, match="slot record"):
            L.call(fn, P(0x10000), 0, 0, 1, 256, P(0x20000), 8, 4, 64, P(0x30000), None)
        with pytest.raises(ValueError, match="slot record"):
            L.call(fn, P(0x10000), 512, 1 << 62, 3, 256, P(0x20000), 8, 4, 64, P(0x30000), None)
    # an empty slot list is a no-op, even with no list pointer
    L.call("gsec_slots_gather", P(0x10000), 512, 256, 1, 256, None, 8, 0, 64, P(0x30000), None)


def test_slots_gather_rejects_host_tensors():
    import torch

    c = pkg("codec")
    pool = torch.zeros(8, 2, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        c.slots_gather(pool, torch.arange(4), torch.empty(4096, dtype=torch.uint8))


def test_copy_gather_argument_checks_run_on_host():
    """Rejected before any launch: source count, a source size that is not a
    multiple of 16, a null source (null pointers only, so nothing is launched)."""
    L = pkg("_lib")
    sizes = (ctypes.c_int64 * 2)(32, 32)
    with pytest.raises(ValueError, match="sources"):
        L.call("gsec_copy_gather", L.ptr_array([0, 0]), sizes, 0, None, None)
    with pytest.raises(ValueError, match="16"):
        L.call("gsec_copy_gather", L.ptr_array([0, 0]), (ctypes.c_int64 * 2)(8, 32), 2, None, None)
    with pytest.raises(ValueError, match="aligned"):
        L.call("gsec_copy_gather", L.ptr_array([0, 0]), sizes, 2, None, None)
    L.call("gsec_copy_gather", L.ptr_array([0]), (ctypes.c_int64 * 1)(0), 1, None, None)  # nothing to copy


@pytest.mark.parametrize("sub", ["xor", "rdp", "rs"])
def test_dropin_demo_runs_as_a_script(sub):
    """The reference runs its demos as `cd benchmark/<code>; python main.py`;
    the drop-ins start the same way (argument parsing needs no GPU)."""
    import subprocess
    import sys

    d = os.path.join(ROOT, "26mlsys-ae-ghostserve_b200", "benchmark", sub)
    r = subprocess.run([sys.executable, "main.py", "--help"], cwd=d, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "--num_data_shards" in r.stdout
