"""The hot kernels compile for sm_100a without register spills (ptxas -v on the
CPU). Guards against changes elsewhere in a translation unit altering their
register allocation, as an inlined helper once did (gf8_fixed_kernel<2,3,7,8>
at 32 registers with spills, RS8 k=3 at 0.63 of HBM instead of 0.89)."""
from __future__ import annotations

import concurrent.futures as cf
import os
import re
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "26mlsys-ae-ghostserve_b200", "csrc")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

HOT = [r"rdp_encode_tma_kernelILi7E", r"rdp_decode_tma_kernelILi7E", r"xor_tma_kernelILi1E",
       r"xor_tma_kernelILi4E"] + [rf"gf8_fixed_kernelILi{k}ELb0E" for k in range(2, 9)] + \
      [rf"gf8_fixed_kernelILi{k}ELb1E" for k in (4, 5)] + \
      [rf"gf8_cauchy_kernelILi{k}ELi{m}ELb{f}E" for k in range(2, 8) for m in (1, 2) if k + m <= 8 for f in (0, 1)]


def ptxas_report(src: str, out_dir: str) -> str:
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
           "-I", os.path.join(ROOT, "include"), "--expt-relaxed-constexpr", "-Xptxas", "-v", "-c",
           os.path.join(CSRC, src), "-o", os.path.join(out_dir, src + ".o")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stderr


@pytest.mark.skipif(not (os.path.exists(NVCC) or shutil.which("nvcc")), reason="nvcc not installed")
def test_hot_kernels_do_not_spill():
    tmp = tempfile.mkdtemp()
    try:
        with cf.ThreadPoolExecutor(2) as ex:
            logs = "".join(ex.map(lambda f: ptxas_report(f, tmp), ["rdp.cu", "linear.cu"]))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    found = {}
    cur = None
    for line in logs.splitlines():
        m = re.search(r"Compiling entry function '(\S+)'", line)
        if m:
            cur = m.group(1)
            continue
        m = re.search(r"(\d+) bytes spill stores", line)
        if m and cur:
            for pat in HOT:
                if re.search(pat, cur):
                    found[pat] = int(m.group(1))
    assert set(found) == set(HOT), set(HOT) - set(found)
    assert all(v == 0 for v in found.values()), found
