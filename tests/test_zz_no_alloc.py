"""qflash_fwd_fused_noalloc (scratch in the library's own device array) gives
the same outputs as qflash_fwd_fused (caller workspace), called through the
C ABI.  Collected last so it also runs after every other test of the session
has used the library; it passes alone in a fresh process too."""
import ctypes

import pytest
import torch

from qflash_b200 import _lib
from qflash_b200 import kernel as K
from qflash_b200.swin import relative_position_index, shifted_window_mask, window_bias

pytestmark = pytest.mark.gpu


def _case(name):
    g = torch.Generator(device="cuda").manual_seed(7)
    if name == "vit_fp16":
        q, k, v = (torch.randn(3, 12, 197, 64, generator=g, device="cuda").half() for _ in range(3))
        return q, k, v, None, 0
    if name == "bool_mask_fp32":
        q, k, v = (torch.randn(2, 4, 130, 128, generator=g, device="cuda") for _ in range(3))
        m = (torch.rand(2, 1, 130, 130, generator=g, device="cuda") > 0.3)
        return q, k, v, m, 0
    # Swin stage-1 shape: per-window float bias with a window period of 16
    heads, nW, N = 3, 16, 49
    q, k, v = (torch.randn(2 * nW, heads, N, 32, generator=g, device="cuda").to(torch.bfloat16) for _ in range(3))
    table = torch.randn(13 * 13, heads, generator=g, device="cuda") * 2
    b = window_bias(table, relative_position_index(7, 7).cuda())
    m = (b + shifted_window_mask(28, 28, 7, 3).cuda()[:, None]).to(torch.bfloat16)  # [nW, heads, N, N]
    return q, k, v, m, nW


def _args(q, k, v, m, period):
    Z, H, N, D = q.shape
    dev = q.device
    q8, k8, v8, o8 = (torch.empty((Z, H, N, D), dtype=torch.int8, device=dev) for _ in range(4))
    out = torch.empty((Z, H, N, D), dtype=q.dtype, device=dev)
    if m is None:
        mask = (None, -1, None, 0, 0, 0)
    else:
        ms = (ctypes.c_int64 * 4)(*[0 if m.shape[i] == 1 else m.stride(i) for i in range(4)])
        mask = (m.data_ptr(), _lib.DTYPES[str(m.dtype)], ms, m.shape[0], m.shape[1], period)
    head = (q.data_ptr(), k.data_ptr(), v.data_ptr(), _lib.DTYPES[str(q.dtype)],
            _lib._strides(q), _lib._strides(k), _lib._strides(v), *mask,
            q8.data_ptr(), k8.data_ptr(), v8.data_ptr(), o8.data_ptr(), out.data_ptr(),
            Z, H, N, D, (1.0 / D ** 0.5) * K.LOG2E, K.L_SHIFT, K.ACC_SHIFT, 0)
    # q8, k8 and v8 are returned too: the call keeps only their raw pointers
    return head, (q8, k8, v8, o8, out)


def _run_workspace(case):
    head, bufs = _args(*case)
    Z, H, N = case[0].shape[:3]
    m = case[3]
    ws_bytes = _lib.fused_workspace_bytes(m.shape[0] if m is not None else 0, m.shape[1] if m is not None else 0, N)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.load().qflash_fwd_fused(*head, ws.data_ptr(), ws.numel(), stream)
    assert rc == 0, _lib.load().qflash_last_error()
    return bufs + (ws,)


def _run_noalloc(case):
    head, bufs = _args(*case)
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.load().qflash_fwd_fused_noalloc(*head, stream)
    assert rc == 0, _lib.load().qflash_last_error()
    return bufs


@pytest.mark.parametrize("name", ["vit_fp16", "bool_mask_fp32", "swin_bf16"])
def test_noalloc_equals_workspace_entry(name):
    case = _case(name)
    ref = _run_workspace(case)
    first = _run_noalloc(case)
    second = _run_noalloc(case)  # the scratch still holds the first call's contents
    torch.cuda.synchronize()
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
    for got in (first, second):
        for a, b in zip(got, ref[:5]):  # q8, k8, v8, o8, out
            assert torch.equal(a, b)  # bit-exact: both entries run the same kernels
    assert not torch.isnan(ref[4].float()).any()
    assert torch.equal(ref[4], K.forward_fused(*case[:4], bias_z_period=case[4]))


def test_noalloc_back_to_back_cases_share_the_scratch():
    cases = [_case("swin_bf16"), _case("vit_fp16")]
    refs = [_run_workspace(c) for c in cases]
    outs = [_run_noalloc(c) for c in cases]  # two calls in a row, different masks and sizes
    torch.cuda.synchronize()
    for got, ref in zip(outs, refs):
        assert all(torch.equal(a, b) for a, b in zip(got, ref[:5]))


def test_noalloc_rejects_a_mask_beyond_the_scratch():
    q, k, v = (torch.randn(64, 12, 197, 64, device="cuda", dtype=torch.float16) for _ in range(3))
    m = torch.zeros(64, 12, 197, 197, device="cuda", dtype=torch.float16)  # 64*12*197*200*4 B of int32 bias
    head, _bufs = _args(q, k, v, m, 0)
    rc = _lib.load().qflash_fwd_fused_noalloc(*head, torch.cuda.current_stream().cuda_stream)
    assert rc == -6  # QFLASH_ERR_UNSUPPORTED
    assert b"scratch" in _lib.load().qflash_last_error()


def test_noalloc_status_reader_and_argument_checks():
    """The no-alloc caller reads the status of its last call through
    qflash_fused_noalloc_status (an all-zero q: status 1, where the reference
    raises ZeroDivisionError); bad mask extents are argument errors."""
    q, k, v = (torch.randn(2, 3, 40, 32, device="cuda") for _ in range(3))
    q.zero_()
    head, _bufs = _args(q, k, v, None, 0)
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.load().qflash_fwd_fused_noalloc(*head, stream) == 0
    st = ctypes.c_int64(-7)
    assert _lib.load().qflash_fused_noalloc_status(q.data_ptr(), stream, ctypes.byref(st)) == 0
    assert st.value == 1
    q2 = torch.randn_like(k)
    head, _bufs = _args(q2, k, v, None, 0)
    assert _lib.load().qflash_fwd_fused_noalloc(*head, stream) == 0
    assert _lib.load().qflash_fused_noalloc_status(q2.data_ptr(), stream, ctypes.byref(st)) == 0
    assert st.value == 0
    m = torch.zeros(2, 3, 40, 40, device="cuda")
    head, _bufs = _args(q2, k, v, m, 0)
    head = list(head)
    head[10] = -1        # mask_zb
    assert _lib.load().qflash_fwd_fused_noalloc(*head, stream) == -1   # QFLASH_ERR_ARG


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_entry_points_restore_the_current_device():
    """A call with data on device 1 while device 0 is current leaves device 0 current."""
    torch.cuda.set_device(0)
    x = torch.randn(1, 2, 64, 32, device="cuda:1")
    head, _bufs = _args(x, x, x, None, 0)
    with torch.cuda.device(1):
        stream = torch.cuda.current_stream().cuda_stream
    assert _lib.load().qflash_fwd_fused_noalloc(*head, stream) == 0
    torch.cuda.synchronize(1)
    assert torch.cuda.current_device() == 0
