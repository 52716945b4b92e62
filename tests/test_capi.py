"""The C-ABI library loads here (no GPU needed) and exports every declared symbol."""
import ctypes
import re
from pathlib import Path


REPO = Path(__file__).resolve().parents[1]


def declared_functions():
    names = []
    for header in sorted((REPO / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names += re.findall(r"\b(anvilq_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_declared_symbols():
    from anvilq_b200 import build, _lib
    build.build()
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name
    # the ctypes binding covers exactly the declared ABI
    assert set(_lib.SIGNATURES) == set(names)


def test_host_only_calls():
    from anvilq_b200 import _lib
    lib = _lib.load()
    assert lib.anvilq_abi_version() == 1
    assert lib.anvilq_strerror(0) == b"ok"
    assert b"workspace" in lib.anvilq_strerror(-4)
    # argument validation happens on the host, before any launch
    assert lib.anvilq_w4a16_gemm(None, None, None, None, None, None, 1, 128, 64, 128, None, 0, None, None) == -1
    assert lib.anvilq_awq_pack(None, None, 1, 8, None) == -1
    assert lib.anvilq_awq_dequant(None, None, None, None, None, 128, 64, 128, None, None) == -1
