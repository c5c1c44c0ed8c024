"""ctypes binding of the C ABI declared in include/qflash_b200.h.

This is the binding a maintainer of the reference would add: plain pointers,
sizes and strides, no torch types crossing the boundary.  The library must be
present (``python -m qflash_b200.build``); there is no fallback.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqflash_b200.so"

FLAG_EXP_IDIV = 1
FLAG_L_IDIV = 2
FLAG_ACC_IDIV = 4
FLAG_DIV_FULL = 8
FLAG_DIV_IEEE = 16

ERRORS = {-1: "QFLASH_ERR_ARG", -2: "QFLASH_ERR_ALIGN", -3: "QFLASH_ERR_TMA", -4: "QFLASH_ERR_LAUNCH",
          -5: "QFLASH_ERR_DEVICE", -6: "QFLASH_ERR_UNSUPPORTED"}

# name -> (restype, argtypes); every symbol the header declares
_I64x4 = ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "qflash_i8_fwd": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        _I64x4, _I64x4, _I64x4, _I64x4, _I64x4,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p]),
    "qflash_i8_fwd_ex": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        _I64x4, _I64x4, _I64x4, _I64x4, _I64x4, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p]),
    "qflash_i8_fwd_gather": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        _I64x4, _I64x4, _I64x4, _I64x4, _I64x4, ctypes.c_int,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
        ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p]),
    "qflash_peer_max": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
        ctypes.c_int, ctypes.c_int, ctypes.c_uint32, ctypes.c_void_p]),
    "qflash_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "qflash_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "qflash_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "qflash_ipc_free": (ctypes.c_int, [ctypes.c_void_p]),
    "qflash_fwd_fused": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, _I64x4, _I64x4, _I64x4,
        ctypes.c_void_p, ctypes.c_int, _I64x4, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "qflash_fwd_fused_out": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, _I64x4, _I64x4, _I64x4,
        ctypes.c_void_p, ctypes.c_int, _I64x4, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _I64x4,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "qflash_fwd_fused_window": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, _I64x4, _I64x4, _I64x4,
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int64 * 2, ctypes.c_int, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _I64x4,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "qflash_fwd_fused_noalloc": (ctypes.c_int, [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, _I64x4, _I64x4, _I64x4,
        ctypes.c_void_p, ctypes.c_int, _I64x4, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_uint32, ctypes.c_void_p]),
    "qflash_fused_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qflash_fused_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]),
    "qflash_device_error": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "qflash_launch_count": (ctypes.c_uint64, []),
    "qflash_last_grid": (ctypes.c_int, []),
    "qflash_version": (ctypes.c_char_p, []),
    "qflash_last_error": (ctypes.c_char_p, []),
    "qflash_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_longlong]),
    "qflash_i8_mma_peak": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "qflash_fused_noalloc_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]),
    "qflash_i8_mma_peak_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
}

_lock = threading.Lock()
_lib = None


class QFlashError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load the library once; raise if it is missing (no CPU path exists)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise QFlashError(f"{LIB_PATH} is missing: build it with `python -m qflash_b200.build`")
                lib = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = lib
    return _lib


def _strides(t) -> ctypes.Array:
    return (ctypes.c_int64 * 4)(*[int(s) for s in t.stride()])


def _check(rc: int, what: str):
    if rc != 0:
        msg = load().qflash_last_error().decode(errors="replace")
        raise QFlashError(f"{what} failed: {ERRORS.get(rc, rc)}: {msg}")


def i8_fwd(q, k, v, o, bias, bias_strides, Z, H, N, D, sm_rscale, exp_M, req_M, l_M, acc_M,
           l_shift, acc_shift, flags, stream, bias_z_period=0, o_peers=None, barrier=None) -> None:
    """Launch the attention kernel on device tensors (no synchronisation).
    ``o_peers``: device addresses (ints) of o's rows in other GPUs' copies of
    the gathered output; ``barrier``: (sig, sig_peers, rank, epoch) of the
    gather barrier inside the kernel (qflash_i8_fwd_gather)."""
    lib = load()
    bs = (ctypes.c_int64 * 4)(*bias_strides) if bias is not None else None
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), bias.data_ptr() if bias is not None else None,
            _strides(q), _strides(k), _strides(v), _strides(o), bs, bias_z_period,
            Z, H, N, D, sm_rscale, exp_M, req_M, l_M, acc_M, l_shift, acc_shift, flags)
    if o_peers or barrier:
        o_peers = list(o_peers or [])
        peers = (ctypes.c_void_p * max(1, len(o_peers)))(*[int(p) for p in o_peers])
        sig, sig_peers, rank, epoch = barrier if barrier else (None, [], 0, 0)
        sp = (ctypes.c_void_p * max(1, len(sig_peers)))(*[int(p) for p in sig_peers])
        _check(lib.qflash_i8_fwd_gather(*args, peers, len(o_peers), sig, sp, rank, epoch, stream),
               "qflash_i8_fwd_gather")
    else:
        _check(lib.qflash_i8_fwd_ex(*args, stream), "qflash_i8_fwd_ex")


IPC_HANDLE_BYTES = 64
SIG_WORDS = 128


def peer_max(inp, out, sig: int, sig_peers, rank: int, epoch: int, stream) -> None:
    """out[:n] = max over the ranks of inp[:n] (float32 device tensors, n <= 4)
    through the ranks' signal words (qflash_peer_max); no synchronisation."""
    sp = (ctypes.c_void_p * max(1, len(sig_peers)))(*[int(p) for p in sig_peers])
    _check(load().qflash_peer_max(inp.data_ptr(), inp.numel(), out.data_ptr(), sig, sp, len(sig_peers), rank, epoch,
                                  stream), "qflash_peer_max")


def ipc_alloc(nbytes: int) -> tuple[int, bytes]:
    """Device memory on the current device that other processes can map:
    (address, 64-byte CUDA IPC handle)."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(load().qflash_ipc_alloc(nbytes, ctypes.byref(ptr), handle), "qflash_ipc_alloc")
    return int(ptr.value), handle.raw


def ipc_open(handle: bytes) -> int:
    """Map another process's qflash_ipc_alloc buffer; returns its address here."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
    ptr = ctypes.c_void_p()
    _check(load().qflash_ipc_open(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(ptr)),
           "qflash_ipc_open")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _check(load().qflash_ipc_close(ptr), "qflash_ipc_close")


def ipc_free(ptr: int) -> None:
    _check(load().qflash_ipc_free(ptr), "qflash_ipc_free")


DTYPES = {"torch.float32": 0, "torch.float16": 1, "torch.bfloat16": 2, "torch.bool": 3}


def fwd_fused(q, k, v, mask, mask_strides, mask_zb, mask_hb, mask_z_period, q8, k8, v8, o8, out,
              scale_log2e, l_shift, acc_shift, flags, workspace, stream) -> None:
    """Launch the on-device forward (qflash_fwd_fused); no synchronisation."""
    lib = load()
    Z, H, N, D = q.shape
    ms = (ctypes.c_int64 * 4)(*mask_strides) if mask is not None else None
    rc = lib.qflash_fwd_fused(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[str(q.dtype)],
                              _strides(q), _strides(k), _strides(v),
                              mask.data_ptr() if mask is not None else None,
                              DTYPES[str(mask.dtype)] if mask is not None else -1, ms, mask_zb, mask_hb, mask_z_period,
                              q8.data_ptr(), k8.data_ptr(), v8.data_ptr(), o8.data_ptr(), out.data_ptr(),
                              Z, H, N, D, scale_log2e, l_shift, acc_shift, flags,
                              workspace.data_ptr(), workspace.numel(), stream)
    _check(rc, "qflash_fwd_fused")


def fwd_fused_out(q, k, v, mask, mask_strides, mask_zb, mask_hb, mask_z_period, q8, k8, v8, out,
                  scale_log2e, l_shift, acc_shift, flags, workspace, stream) -> None:
    """Launch qflash_fwd_fused_out: the epilogue writes ``out`` (any strides,
    head dim contiguous) directly; no synchronisation."""
    lib = load()
    Z, H, N, D = q.shape
    ms = (ctypes.c_int64 * 4)(*mask_strides) if mask is not None else None
    rc = lib.qflash_fwd_fused_out(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[str(q.dtype)],
                                  _strides(q), _strides(k), _strides(v),
                                  mask.data_ptr() if mask is not None else None,
                                  DTYPES[str(mask.dtype)] if mask is not None else -1, ms, mask_zb, mask_hb,
                                  mask_z_period, q8.data_ptr(), k8.data_ptr(), v8.data_ptr(), out.data_ptr(),
                                  _strides(out), Z, H, N, D, scale_log2e, l_shift, acc_shift, flags,
                                  workspace.data_ptr(), workspace.numel(), stream)
    _check(rc, "qflash_fwd_fused_out")


def fwd_fused_window(q, k, v, table, index, window_mask, num_windows, q8, k8, v8, out,
                     scale_log2e, l_shift, acc_shift, flags, workspace, stream) -> None:
    """Launch qflash_fwd_fused_window (Swin bias built on the device)."""
    lib = load()
    Z, H, N, D = q.shape
    ts = (ctypes.c_int64 * 2)(int(table.stride(0)), int(table.stride(1)))
    rc = lib.qflash_fwd_fused_window(q.data_ptr(), k.data_ptr(), v.data_ptr(), DTYPES[str(q.dtype)],
                                     _strides(q), _strides(k), _strides(v),
                                     table.data_ptr(), DTYPES[str(table.dtype)], ts, int(table.shape[0]),
                                     index.data_ptr(),
                                     window_mask.data_ptr() if window_mask is not None else None,
                                     DTYPES[str(window_mask.dtype)] if window_mask is not None else -1,
                                     num_windows, q8.data_ptr(), k8.data_ptr(), v8.data_ptr(), out.data_ptr(),
                                     _strides(out), Z, H, N, D, scale_log2e, l_shift, acc_shift, flags,
                                     workspace.data_ptr(), workspace.numel(), stream)
    _check(rc, "qflash_fwd_fused_window")


def fused_workspace_bytes(mask_zb: int, mask_hb: int, N: int) -> int:
    return int(load().qflash_fused_workspace_bytes(mask_zb, mask_hb, N))


def fused_status(workspace, stream) -> int:
    out = ctypes.c_int64(0)
    _check(load().qflash_fused_status(workspace.data_ptr(), stream, ctypes.byref(out)), "qflash_fused_status")
    return int(out.value)


def device_error(stream) -> int:
    out = ctypes.c_uint32(0)
    _check(load().qflash_device_error(stream, ctypes.byref(out)), "qflash_device_error")
    return int(out.value)


def launch_count() -> int:
    return int(load().qflash_launch_count())


def last_grid() -> int:
    return int(load().qflash_last_grid())


def i8_mma_peak_tops(ctas_per_sm: int = 1, iters: int = 20000, reps: int = 5) -> float:
    """Measured dense int8 tensor-core throughput of the current GPU in TOPS
    (best of `reps` timed launches of qflash_i8_mma_peak, CUDA events)."""
    import torch
    stream = torch.cuda.current_stream()
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    _check(load().qflash_i8_mma_peak(ctas_per_sm, iters, stream.cuda_stream), "qflash_i8_mma_peak")  # warm-up
    best = float("inf")
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _check(load().qflash_i8_mma_peak(ctas_per_sm, iters, stream.cuda_stream), "qflash_i8_mma_peak")
        e1.record(stream)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    err = ctypes.c_uint32(0)
    _check(load().qflash_i8_mma_peak_status(stream.cuda_stream, ctypes.byref(err)), "qflash_i8_mma_peak_status")
    if err.value:
        raise QFlashError("the int8 MMA peak kernel's wait gave up")
    ops = sms * ctas_per_sm * iters * 2.0 * 128 * 256 * 32
    return ops / (best * 1e-3) / 1e12
