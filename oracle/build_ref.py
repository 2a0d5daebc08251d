"""Build recipe for ``oracle/_ref``: the reference's own CUDA extensions, compiled
from the reference sources where they lie, for use as a parity checker only.

This is test infrastructure. Nothing in the product imports it; only ``tests/``,
``__graft_entry__.smoke()`` and the golden-vector generator load what it builds.

What it builds (one torch extension per reference source, same module names the
reference's own ``torch.utils.cpp_extension.load`` calls use):

* ``xor_kernel``               from ``benchmark/xor/kernel.cu``  (``benchmark/xor/main.py:29-35``)
* ``rdp_kernel_rdp_parallel``  from ``benchmark/rdp/kernel.cu``  (``benchmark/rdp/main.py:34-40``)
* ``rs_kernel16``              from ``benchmark/rs/kernel.cu``   (``benchmark/rs/main.py:27-33``)
* ``rdp_kv_ops``               from the ``CUDA_RDP_SRC`` string in ``bench_ghostserve_rdp.py:92-207``
  (the reference JIT-writes that string to a temp ``.cu`` file, ``:272-283``; this recipe does the
  same, into ``oracle/_ref/rdp_kv_ops/``, which is git-ignored).

The reference sets no B200 architecture, so the arch list is set to ``10.0`` here;
the compile flags are the ones each reference ``load`` call passes.

Outputs go only under ``oracle/_ref/``. The reference tree is read-only and only
present in the build container; on a GPU box the prebuilt ``.so`` files travel
with the repository snapshot and are loaded by :func:`load_ref`.
"""
from __future__ import annotations

import ast
import importlib.machinery
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
# The reference checkout: $GSEC_REFERENCE_ROOT, else a directory named
# "reference" beside this repository's root.
REF_ROOT_DEFAULT = os.environ.get("GSEC_REFERENCE_ROOT") or os.path.normpath(
    os.path.join(HERE, os.pardir, os.pardir, "reference"))

# (module name, source path relative to the reference root or None for the hook string, cuda flags)
REF_EXTS = {
    "xor_kernel": ("benchmark/xor/kernel.cu", ["--expt-relaxed-constexpr", "--use_fast_math"]),
    "rdp_kernel_rdp_parallel": ("benchmark/rdp/kernel.cu",
                                ["--expt-relaxed-constexpr", "--use_fast_math", "-lineinfo"]),
    "rs_kernel16": ("benchmark/rs/kernel.cu",
                    ["--expt-relaxed-constexpr", "--use_fast_math", "-lineinfo"]),
    "rdp_kv_ops": (None, ["-O3"]),
}


def _hook_source(ref_root: str) -> str:
    """Return the CUDA source string the reference hook compiles at run time."""
    path = os.path.join(ref_root, "bench_ghostserve_rdp.py")
    tree = ast.parse(open(path, encoding="utf-8").read())
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
                isinstance(t, ast.Name) and t.id == "CUDA_RDP_SRC" for t in node.targets):
            return ast.literal_eval(node.value)
    raise RuntimeError("CUDA_RDP_SRC not found in bench_ghostserve_rdp.py")


def _so_path(name: str) -> str:
    return os.path.join(REF_OUT, name, name + ".so")


def built(name: str) -> bool:
    return os.path.exists(_so_path(name))


def build(ref_root: str = REF_ROOT_DEFAULT, names=None, verbose: bool = False) -> list:
    """Compile the reference extensions that are not built yet. Returns built names."""
    if not os.path.isdir(ref_root):
        return []
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    from torch.utils.cpp_extension import load  # noqa: WPS433 (heavy import kept local)

    done = []
    for name, (rel, flags) in REF_EXTS.items():
        if names is not None and name not in names:
            continue
        if built(name):
            done.append(name)
            continue
        bdir = os.path.join(REF_OUT, name)
        os.makedirs(bdir, exist_ok=True)
        if rel is None:
            src = os.path.join(bdir, name + ".cu")
            with open(src, "w", encoding="utf-8") as f:
                f.write(_hook_source(ref_root))
        else:
            src = os.path.join(ref_root, rel)
        load(name=name, sources=[src], extra_cuda_cflags=list(flags),
             extra_cflags=["-std=c++17"] if rel is not None else ["-O3"],
             build_directory=bdir, verbose=verbose, with_cuda=True)
        done.append(name)
    return done


def load_ref(name: str):
    """Import a prebuilt reference extension from ``oracle/_ref`` (no compilation)."""
    if name in sys.modules:
        return sys.modules[name]
    path = _so_path(name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"reference extension {name} not built at {path}")
    import torch  # noqa: F401  (resolves libtorch symbols the extension links against)
    loader = importlib.machinery.ExtensionFileLoader(name, path)
    spec = importlib.util.spec_from_file_location(name, path, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
