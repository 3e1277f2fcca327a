"""CPU-side checks of the C ABI: the library builds for sm_100a, loads, and exports every entry
point include/slx.h declares. No device calls (this container has no GPU)."""
import ctypes
import os

import pytest

from spatialdb_b200 import _lib, build


def test_library_builds_and_exports_header_symbols():
    path = build.build()
    assert os.path.exists(path)
    cdll = ctypes.CDLL(path)
    declared = _lib.header_symbols()
    assert len(declared) >= 15
    missing = [s for s in declared if not hasattr(cdll, s)]
    assert not missing, f"declared in slx.h but not exported: {missing}"


def test_binding_table_matches_header():
    declared = set(_lib.header_symbols())
    assert declared == set(_lib.SIGNATURES), (declared ^ set(_lib.SIGNATURES))


def test_version_string_without_device():
    lib = _lib.lib()
    assert lib.slx_version().decode().startswith("slx")


def test_product_sources_do_not_reference_oracle():
    """The product path never loads the oracle (it is test infrastructure)."""
    root = os.path.dirname(build.PKG)
    for dirpath, _, files in os.walk(build.PKG):
        if "_build" in dirpath:
            continue
        for f in files:
            if f.endswith((".py", ".cu", ".cpp", ".h", ".cuh", ".hpp")):
                src = open(os.path.join(dirpath, f), errors="replace").read()
                assert "import oracle" not in src and "slx_oracle" not in src and "libslx_oracle" not in src, f
    assert os.path.isdir(os.path.join(root, "oracle"))
