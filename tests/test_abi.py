"""CPU checks of the product library: it builds for sm_100a, loads, and exports
every entry point include/czg.h declares (no compute calls without a GPU)."""
import ctypes
import os
import re


def test_library_exports_header_symbols(root):
    from compress_zip_b200 import build, engine

    build.build()
    hdr = open(os.path.join(root, "include", "czg.h")).read()
    declared = set(re.findall(r"\b(czg_[a-z0-9_]+)\s*\(", hdr))
    assert declared, "no entry points parsed from include/czg.h"
    lib = ctypes.CDLL(engine.LIB_PATH)
    for name in sorted(declared):
        assert hasattr(lib, name), f"{name} declared in czg.h but not exported"
    assert declared == set(engine.EXPORTS)


def test_compress_bound():
    from compress_zip_b200 import engine

    L = engine.lib()
    assert L.czg_compress_bound(0, 0) == 0
    assert L.czg_compress_bound(1024, 1) == 4 * 1024 + 8
