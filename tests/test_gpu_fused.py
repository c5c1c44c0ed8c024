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
