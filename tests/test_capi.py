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


def test_python_constants_match_header():
    """Status codes, quantiser modes and operand kinds: the Python binding's
    values are the header's."""
    txt = open(os.path.join(ROOT, "include", "boa_b200.h")).read()
    defs = dict(re.findall(r"#define\s+(BOA_(?:OK|ERR_\w+|QUANT_\w+|WEIGHTS_\w+))\s+(\d+)", txt))
    assert len(defs) >= 14
    for name, value in defs.items():
        assert getattr(_native, name) == int(value), name
    import model
    import boa_b200.container as C
    # every operand kind has a Python name and a container code
    assert set(model.WEIGHT_FORMATS.values()) == {int(v) for k, v in defs.items() if k.startswith("BOA_WEIGHTS_")}
    assert set(C.WEIGHT_FORMAT_CODES) == set(model.WEIGHT_FORMATS)
