"""Build the reference's own CUDA range coder into ``oracle/_ref/`` (test pin).

The reference embeds its batched coder as a CUDA source string inside
``gpu_range_coder.py`` (lines 26-325) and compiles it with nvcc + pybind11 at
import time (lines 327-375).  This recipe does the same compile, unmodified,
from the file where it lies under the reference tree, but adds
``-gencode arch=compute_100a,code=sm_100a`` (the reference passes no arch) and
writes only the resulting extension module into ``oracle/_ref/`` (git-ignored;
it travels to the GPU box with the snapshot).  The extracted source goes to a
temporary directory and is deleted afterwards; nothing from the reference is
copied into the repository.

On the GPU box ``tests/test_ref_pin.py`` loads this module and checks the C
oracle (``oracle/rc_oracle.c``) against it bit for bit at PRECISION 24.

Usage: python oracle/build_ref.py [--reference /path/to/reference]
Skips (exit 0, message) when the reference tree is absent, e.g. on the GPU box.
"""
from __future__ import annotations

import argparse
import ast
import os
import shutil
import subprocess
import sys
import sysconfig
import tempfile
from importlib.machinery import EXTENSION_SUFFIXES

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MOD_NAME = "_gpu_range_cuda_ext"


def _extract_cuda_source(py_path: str) -> str:
    tree = ast.parse(open(py_path, encoding="utf-8").read())
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == "cuda_code"
                                                for t in node.targets):
            call = node.value  # dedent(r'''...''')
            if isinstance(call, ast.Call) and call.args and isinstance(call.args[0], ast.Constant):
                import textwrap
                return textwrap.dedent(call.args[0].value)
    raise RuntimeError(f"cuda_code string not found in {py_path}")


def module_path() -> str:
    return os.path.join(OUT_DIR, MOD_NAME + EXTENSION_SUFFIXES[0])


def reference_root() -> str | None:
    """Where the reference checkout is: $BOA_REFERENCE_ROOT, else a directory
    named ``reference`` beside this repository's root (a sibling checkout);
    None when neither exists (e.g. on a GPU box, which uses the prebuilt
    module)."""
    env = os.environ.get("BOA_REFERENCE_ROOT")
    if env:
        return env if os.path.isdir(env) else None
    sib = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "reference")
    return sib if os.path.isdir(sib) else None


def build(reference: str | None = None, force: bool = False) -> str | None:
    reference = reference or reference_root()
    if not reference:
        print("[build_ref] no reference checkout found ($BOA_REFERENCE_ROOT unset, no sibling 'reference'); skipping")
        return None
    src_py = os.path.join(reference, "gpu_range_coder.py")
    if not os.path.exists(src_py):
        print(f"[build_ref] reference not present at {reference}; skipping")
        return None
    out = module_path()
    if os.path.exists(out) and not force and os.path.getmtime(out) >= os.path.getmtime(src_py):
        return out
    import pybind11
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = tempfile.mkdtemp(prefix="boa_ref_build_")
    try:
        cu = os.path.join(tmp, MOD_NAME + ".cu")
        with open(cu, "w", encoding="utf-8") as f:
            f.write(_extract_cuda_source(src_py))
        incs = []
        for k in ("include", "platinclude"):
            p = sysconfig.get_paths().get(k)
            if p and p not in incs:
                incs.append(p)
        for p in (pybind11.get_include(False), pybind11.get_include(True)):
            if p and p not in incs:
                incs.append(p)
        nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
        cmd = [nvcc, cu, "-shared", "-Xcompiler", "-fPIC", "-o", out, "-std=c++17", "-O3",
               "-gencode", "arch=compute_100a,code=sm_100a", "-lcudart"]
        for p in incs:
            cmd += ["-I", p]
        subprocess.check_call(cmd)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return out


def load():
    """Import the built reference module (GPU box / tests only)."""
    import importlib.util
    p = module_path()
    if not os.path.exists(p):
        return None
    spec = importlib.util.spec_from_file_location(MOD_NAME, p)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (default: see reference_root())")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    r = build(a.reference, a.force)
    print(r or "skipped")
    sys.exit(0)
