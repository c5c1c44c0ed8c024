"""forward_fused (qflash_fwd_fused: scales, constants, quantisation, bias and
dequantisation on the device) equals the torch-op host path bit for bit."""
import pytest
import torch

from qflash_b200 import kernel as K
from qflash_b200.swin import relative_position_index, shifted_window_mask, window_bias, window_attn_mask
from qflash_b200.workloads import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("wname,Z", [("vit_b", 3), ("deit_t", 8), ("vit_l", 1)])
def test_fused_equals_host_path(dtype, wname, Z):
    w = WORKLOADS[wname].scaled(Z)
    q, k, v, _ = make_inputs(w, seed=11, device="cuda", dtype=dtype)
    ref = K.forward_with_scales(q, k, v)
    out, (q8, k8, v8, o8) = K.forward_fused(q, k, v, return_int8=True)
    qs, ks, vs = K.tensor_scales(q, k, v)
    assert torch.equal(q8, K.quantize(q, qs)) and torch.equal(v8, K.quantize(v, vs))
    assert out.dtype == ref.dtype and torch.equal(out, ref)


@pytest.mark.parametrize("dtype", DTYPES)
def test_fused_float_and_bool_masks(dtype):
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(4, 3, 70, 64, generator=g, device="cuda").to(dtype) for _ in range(3))
    fm = torch.randn(4, 1, 70, 70, generator=g, device="cuda") * 40
    fm = torch.where(fm > 60, torch.full_like(fm, -100.0), fm)
    fm = torch.where(fm < -70, torch.full_like(fm, -1000.0), fm).to(dtype)
    assert torch.equal(K.forward_fused(q, k, v, fm), K.forward_with_scales(q, k, v, fm))
    bm = torch.rand(70, 70, generator=g, device="cuda") > 0.2
    assert torch.equal(K.forward_fused(q, k, v, bm), K.forward_with_scales(q, k, v, bm))


def test_fused_window_period_and_permuted_inputs():
    torch.manual_seed(0)
    table = torch.randn(169, 6, device="cuda") * 0.02
    idx = relative_position_index(7, 7).cuda()
    mask = shifted_window_mask(28, 28, 7, 3).cuda()                   # 16 windows
    qkv = torch.randn(32, 49, 3, 6, 32, device="cuda").permute(2, 0, 3, 1, 4)   # QAttention-style views
    q, k, v = qkv.unbind(0)
    rel = window_bias(table, idx)
    compact = rel + mask.view(16, 1, 49, 49)
    full = window_attn_mask(table, idx, 2, mask)
    expect = K.forward_with_scales(q, k, v, full)
    assert torch.equal(K.forward_fused(q, k, v, compact, bias_z_period=16), expect)
    assert torch.equal(K.forward_fused(q, k, v, full), expect)


def test_fused_zero_input_reports_like_reference():
    q = torch.zeros(1, 2, 40, 32, device="cuda")
    k = torch.randn(1, 2, 40, 32, device="cuda")
    with pytest.raises(ZeroDivisionError):
        K.forward_with_scales(q, k, k)
    with pytest.raises(ZeroDivisionError):
        K.forward_fused(q, k, k, check=True)
    assert torch.isnan(K.forward_fused(q, k, k)).all()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_epilogue_output_equals_int8_path(dtype, D):
    """The attention epilogue writing o8 * o_scale itself (qflash_fwd_fused_out)
    gives the same bits as the int8 output plus the separate dequantisation."""
    g = torch.Generator(device="cuda").manual_seed(D)
    q, k, v = (torch.randn(3, 4, 130, D, generator=g, device="cuda").to(dtype) for _ in range(3))
    direct = K.forward_fused(q, k, v)
    via_int8, _ = K.forward_fused(q, k, v, return_int8=True)
    assert torch.equal(direct, via_int8)
    assert torch.equal(direct, K.forward_with_scales(q, k, v))


@pytest.mark.parametrize("dtype", DTYPES)
def test_epilogue_output_into_permuted_buffer(dtype):
    """A [Z, N, H, D] buffer seen as [Z, H, N, D] (QAttention's reshape target)
    receives the same values; the rows are 16-byte aligned or not."""
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(2, 6, 197, 64, generator=g, device="cuda").to(dtype) for _ in range(3))
    expect = K.forward_with_scales(q, k, v)
    buf = torch.full((2, 197, 6, 64), 7.0, device="cuda", dtype=dtype)
    K.forward_fused(q, k, v, out=buf.permute(0, 2, 1, 3))
    assert torch.equal(buf.permute(0, 2, 1, 3), expect)
    # an odd element offset: no 16-byte vector stores
    big = torch.full((2 * 197 * 6 * 64 + 1,), 7.0, device="cuda", dtype=dtype)
    view = big[1:].view(2, 197, 6, 64).permute(0, 2, 1, 3)
    K.forward_fused(q, k, v, out=view)
    assert torch.equal(view, expect) and big[0].item() == 7.0


def test_fused_rejects_mismatched_shapes():
    q = torch.randn(1, 2, 70, 64, device="cuda")
    k = torch.randn(1, 2, 64, 64, device="cuda")
    with pytest.raises(ValueError):
        K.forward_fused(q, k, k)


def test_epilogue_output_nan_on_error_status():
    q = torch.zeros(1, 2, 40, 32, device="cuda")
    k = torch.randn(1, 2, 40, 32, device="cuda")
    buf = torch.zeros(1, 40, 2, 32, device="cuda")
    K.forward_fused(q, k, k, out=buf.permute(0, 2, 1, 3))
    assert torch.isnan(buf).all()


def test_qattention_fused_layout_matches_reference_path(monkeypatch):
    from qflash_b200.attention import QAttention
    torch.manual_seed(0)
    m = QAttention(384, 6).cuda().half()
    x = torch.randn(4, 197, 384, device="cuda", dtype=torch.half)
    ref = m(x)
    monkeypatch.setattr(K, "FUSED", True)
    assert torch.equal(m(x), ref)


@pytest.mark.parametrize("dtype", DTYPES)
def test_fused_unaligned_inputs(dtype):
    """Inputs whose rows are not 16-byte aligned take the scalar amax /
    quantisation kernels; aligned ones the vectorised ones: same bits."""
    g = torch.Generator(device="cuda").manual_seed(9)
    shape = (2, 3, 77, 64)
    n = 2 * 3 * 77 * 64
    bufs = [torch.randn(n + 1, generator=g, device="cuda").to(dtype) for _ in range(3)]
    q, k, v = (b[1:].view(shape) for b in bufs)          # element offset 1: misaligned rows
    qa, ka, va = (t.clone() for t in (q, k, v))           # aligned copies
    expect = K.forward_with_scales(q, k, v)
    assert torch.equal(K.forward_fused(q, k, v), expect)
    assert torch.equal(K.forward_fused(qa, ka, va), expect)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantise_every_16bit_value(dtype):
    """The on-device quantisation (reciprocal + FMA residual division for 16-bit
    inputs) against torch's round(x / s) for every finite 16-bit x below a
    range of maxima (each maximum sets the scale s = amax / 127)."""
    bits = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(dtype)
    allv = bits[torch.isfinite(bits.float())].cuda()
    g = torch.Generator(device="cuda").manual_seed(1)
    # maxima whose scale amax / 127 is non-zero in both dtypes (below about
    # 3.8e-6 it is 0 in fp16: the ZeroDivisionError case); 5e-4 and 2e-3 give
    # subnormal fp16 scales, where |x / s| can pass 127.5 and the clamp acts
    maxima = [5e-4, 2e-3, 0.01, 0.37, 0.7, 1.0, 5.5, 127.0, 3.1e3, 6.0e4]
    if dtype == torch.bfloat16:
        # scales outside [2^-96, 2^96] take the IEEE division path
        maxima += [1e-30, 1e35]
    for amax in maxima:
        a = torch.tensor(amax, dtype=dtype, device="cuda")
        x = allv[allv.abs() <= a]
        x = torch.cat([x, a.view(1)])
        n = (x.numel() + 63) // 64 * 64
        q = torch.zeros(n, dtype=dtype, device="cuda")
        q[: x.numel()] = x
        q = q.view(1, 1, n // 64, 64)
        # K scaled by 1 / amax keeps q_scale * k_scale moderate (a valid forward)
        kv = (torch.randn(q.shape, generator=g, device="cuda") / amax).to(dtype)
        _, (q8, _, _, _) = K.forward_fused(q, kv, kv, check=True, return_int8=True)
        qs, _, _ = K.tensor_scales(q, kv, kv)
        assert torch.equal(q8, K.quantize(q, qs)), amax
