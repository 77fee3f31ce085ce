"""The C-ABI library builds, loads and exports every symbol the header declares (no GPU)."""
import os
import re

from miniserve_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "mssample.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ms_[a-z0-9_]+)\s*\(", text)))


def test_builds_and_exports_declared_symbols():
    build.build()
    L = _lib.lib()
    names = declared_functions()
    assert "ms_sample" in names
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, n
    assert L.ms_version() >= 100
    assert L.ms_error_string(-1).decode().startswith("invalid")
