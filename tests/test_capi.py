"""The C-ABI library loads and exports every symbol include/boa_b200.h declares
(no compute calls, no GPU needed)."""
import os
import re

from boa_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "boa_b200.h")).read()
    return set(re.findall(r"BOA_API\s+[\w\s\*]+?\b(boa_\w+)\s*\(", txt))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "boa_rc_create" in syms and "boa_codec_encode" in syms and len(syms) >= 20


def test_library_exports_all_declared_symbols():
    lib = _native.load()
    missing = [s for s in declared_symbols() if getattr(lib, s, None) is None]
    assert not missing, f"missing exports: {missing}"
    assert lib.boa_abi_version() == 1


def test_bindings_cover_header():
    assert declared_symbols() <= set(_native.SIGNATURES)
