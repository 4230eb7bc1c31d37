"""The ctypes binding (specdec_b200) against include/specdec.h, on the CPU:
every declared entry point is bound with as many argument types as the header
gives it parameters (a mismatch would pass garbage through the C ABI)."""
import os
import re

import specdec_b200 as sd

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declarations():
    with open(os.path.join(ROOT, "include", "specdec.h")) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(specdec_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p for p in m.group(2).split(",") if p.strip() and p.strip() != "void"]
        out[m.group(1)] = len(params)
    return out


def test_every_export_is_declared():
    decl = _declarations()
    assert set(sd.EXPORTS) == set(decl), set(sd.EXPORTS) ^ set(decl)


def test_argtypes_match_the_header():
    lib = sd.load_library()
    for name, n in _declarations().items():
        fn = getattr(lib, name)
        assert fn.argtypes is not None, name
        assert len(fn.argtypes) == n, (name, len(fn.argtypes), n)
