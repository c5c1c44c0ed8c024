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


def test_multi_gpu_entry_points_reject_bad_arguments_without_gpu():
    """The gathered-output, scale-exchange and IPC entry points check their
    arguments before any CUDA call."""
    from qflash_b200 import _lib
    lib = _lib.load()
    st = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    peers = (ctypes.c_void_p * 8)()
    # more peer copies than the epilogue takes
    rc = lib.qflash_i8_fwd_gather(None, None, None, None, None, st, st, st, st, None, 0, 1, 1, 8, 64,
                                  100, -5, 500, 1000, 1000, 30, 30, 0, peers, 8, None, None, 0, 1, None)
    assert rc == -1 and b"n_peers" in lib.qflash_last_error()
    # signal words without the peers' signal words
    rc = lib.qflash_i8_fwd_gather(None, None, None, None, None, st, st, st, st, None, 0, 1, 1, 8, 64,
                                  100, -5, 500, 1000, 1000, 30, 30, 0, peers, 1, 16, None, 0, 1, None)
    assert rc == -1 and b"signal" in lib.qflash_last_error()
    x = ctypes.c_float(0.0)
    for n, n_peers, rank, epoch in ((0, 1, 0, 1), (5, 1, 0, 1), (1, 8, 0, 1), (1, 1, 2, 1), (1, 1, 0, 0)):
        rc = lib.qflash_peer_max(ctypes.addressof(x), n, ctypes.addressof(x), 16, peers, n_peers, rank, epoch,
                                 None)
        assert rc == -1 and b"peer_max" in lib.qflash_last_error(), (n, n_peers, rank, epoch)
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    assert lib.qflash_ipc_alloc(0, ctypes.byref(ptr), handle) == -1
    assert lib.qflash_ipc_open(None, ctypes.byref(ptr)) == -1
    assert lib.qflash_ipc_close(None) == -1 and lib.qflash_ipc_free(None) == -1
