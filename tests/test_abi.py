"""The C-ABI library loads and exports every function include/qflash_b200.h declares (no GPU needed)."""
import ctypes
import re

from conftest import ROOT

HEADER = ROOT / "include" / "qflash_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(qflash_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "qflash_i8_fwd" in names and "qflash_device_error" in names


def test_library_exports_every_declared_symbol():
    from qflash_b200 import _lib
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_version_and_argument_errors_without_gpu():
    from qflash_b200 import _lib
    lib = _lib.load()
    assert b"sm_100a" in lib.qflash_version()
    st = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    # bad head dim is rejected before any CUDA call
    rc = lib.qflash_i8_fwd(None, None, None, None, None, st, st, st, st, None, 1, 1, 8, 48,
                           100, -5, 500, 1000, 1000, 30, 30, 0, None)
    assert rc == -1 and b"head dim" in lib.qflash_last_error()
    # empty problems are a no-op
    rc = lib.qflash_i8_fwd(None, None, None, None, None, st, st, st, st, None, 0, 1, 8, 64,
                           100, -5, 500, 1000, 1000, 30, 30, 0, None)
    assert rc == 0
    rc = lib.qflash_i8_fwd(None, None, None, None, None, st, st, st, st, None, 1, 1, 8, 64,
                           100, -5, 500, 1000, 1000, 30, 30, 0, None)
    assert rc == -1 and b"null" in lib.qflash_last_error()
