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


def test_every_entry_point_rejects_null_pointers_on_the_host():
    """Every launching entry point checks its required pointers before touching
    the device: all-null arguments return ANVILQ_EINVAL.  (Run only where no
    GPU is visible, so that a missing check could never launch on null.)"""
    import torch
    if torch.cuda.is_available():
        import pytest
        pytest.skip("host-only check")
    from anvilq_b200 import _lib
    lib = _lib.load()
    P, I, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
    checked = 0
    for name, (res, args) in _lib.SIGNATURES.items():
        if res is not I or P not in args:
            continue
        pointer = lambda a: a is P or (isinstance(a, type) and issubclass(a, ctypes._Pointer))
        vals = [None if pointer(a) else 128 if a is I else 1.0 if a is F else (1 << 20) if a is SZ else 0
                for a in args]
        assert getattr(lib, name)(*vals) == -1, name
        checked += 1
    assert checked >= 30
