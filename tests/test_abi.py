"""The C-ABI library loads on a CPU-only host and exports every symbol include/omq_b200.h declares
(no compute calls: there is no GPU here)."""
import ctypes
import os
import re

from conftest import REPO


def _declared():
    src = open(os.path.join(REPO, "include", "omq_b200.h")).read()
    return sorted(set(re.findall(r"OMQ_API\s+[\w\s\*]+?\b(omq_\w+)\s*\(", src)))


def test_header_declares_api():
    names = _declared()
    assert "omq_engine_create" in names and "omq_search_synthetic" in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol():
    from omoknuni_quantum_b200 import build_ext, _lib
    build_ext.build()
    L = ctypes.CDLL(build_ext.LIB)
    missing = [n for n in _declared() if not hasattr(L, n)]
    assert not missing, missing
    # the Python binding declares a signature for each of them
    assert set(_declared()) <= set(_lib.SIGNATURES)


def test_status_strings_without_gpu():
    from omoknuni_quantum_b200 import _lib
    L = _lib.load()
    assert L.omq_status_string(1) == b"tree full"
    assert L.omq_status_string(0) == b"ok"


def test_struct_layouts_match_the_library():
    """The Python ctypes structures have the sizes the library was compiled with (host call)."""
    import ctypes
    from omoknuni_quantum_b200 import _lib
    e, r = ctypes.c_uint32(), ctypes.c_uint32()
    assert _lib.load().omq_abi_struct_sizes(ctypes.byref(e), ctypes.byref(r)) == 0
    assert e.value == ctypes.sizeof(_lib.EngineConfig)
    assert r.value == ctypes.sizeof(_lib.ResNetConfig)
