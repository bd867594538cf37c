"""The C-ABI library loads on CPU-only hosts and exports every function include/*.h
declares; the ctypes binding covers the same set (no compute calls here)."""
import ctypes
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions() -> set[str]:
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", src, flags=re.M):
            name = m.group(1)
            if name not in ("if", "defined"):
                names.add(name)
    return names


@pytest.fixture(scope="module")
def lib():
    from moe_offload_b200 import _lib
    if not os.path.exists(_lib.LIB_PATH):
        pytest.fail(f"{_lib.LIB_PATH} not built (run __graft_entry__.build())")
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_symbols_exported(lib):
    names = declared_functions()
    assert len(names) >= 5
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_matches_header():
    from moe_offload_b200 import _lib
    names = declared_functions()
    assert names == set(_lib.SIGNATURES), (names ^ set(_lib.SIGNATURES))


def test_version_and_error_without_gpu(lib):
    from moe_offload_b200 import _lib
    L = _lib.load()
    assert L.moe_version() >= 100
    # argument validation happens before any CUDA call, so it works on a CPU-only host
    with pytest.raises(_lib.MoeError) as ei:
        _lib.call("moe_experts_gateup", None, 1, 3072, 768, 10, 512, None, None, None, None, None,
                  None, None, 3, 64, 1, None, None)
    assert "bits=2" in str(ei.value)
