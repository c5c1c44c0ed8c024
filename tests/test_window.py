"""Swin path: the per-window bias (window_attention, QWindowAttention) against
the reference's expanded bias and output."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from qflash_b200 import kernel as K
from qflash_b200.swin import relative_position_index, shifted_window_mask, window_attn_mask, window_bias


def _swin_parts(seed, images, heads, windows):
    """The table / mask generator tests/golden/gen_golden.py used for the cfg4 cases."""
    g = torch.Generator().manual_seed(seed + 1000)
    table = torch.randn((169, heads), generator=g) * 0.02
    idx = relative_position_index(7, 7)
    mask = None
    if windows > 1:
        side = int(round(windows ** 0.5)) * 7
        mask = shifted_window_mask(side, side, 7, 3)
    return table, idx, mask


def test_window_bias_equals_expanded_reference_bias(golden):
    rec = golden("cfg4_swin_s1")
    table, idx, mask = _swin_parts(4, 2, 3, 4)
    full = window_attn_mask(table, idx, 2, mask)
    assert torch.equal(full, torch.from_numpy(rec["mask"]))        # same generator as the fixture
    Z, H, N, _ = rec["q8"].shape
    sm_scale, *_ = K.fixed_point_params(float(rec["qk_scale"]), 32, None)
    rel = window_bias(table, idx)
    bias, st = K.quantize_bias(rel + mask.view(4, 1, N, N), sm_scale, 4, H, N)
    per_window = torch.as_strided(bias, (4, H, N, N), st).numpy()
    for b in range(Z):
        np.testing.assert_array_equal(per_window[b % 4], rec["bias"][b])


def test_shifted_window_mask_regions():
    m = shifted_window_mask(14, 14, 7, 3)
    assert m.shape == (4, 49, 49)
    assert torch.all(m[0] == 0)                      # top-left window: one region
    assert set(m.unique().tolist()) == {0.0, -100.0}
    assert torch.equal(m, m.transpose(1, 2))


@pytest.mark.gpu
def test_window_attention_matches_reference_output(golden):
    rec = golden("cfg4_swin_s1")
    table, idx, mask = _swin_parts(4, 2, 3, 4)
    q, k, v = (torch.from_numpy(rec[x]).cuda() for x in "qkv")
    out = K.window_attention(q, k, v, window_bias(table, idx).cuda(), mask.cuda())
    # the default final division is the one of the reference's compiled kernel on B200
    with np.load(GOLDEN / "triton_gpu" / "cfg4_swin_s1.npz") as z:
        o8 = z["o8"]
    expect = torch.from_numpy(o8).cuda() * (v.abs().amax() / 127)
    assert torch.equal(out, expect)


@pytest.mark.gpu
@pytest.mark.parametrize("images,windows,heads", [(3, 4, 3), (2, 16, 6), (5, 1, 24)])
def test_window_attention_equals_full_mask_path(images, windows, heads):
    table, idx, mask = _swin_parts(7 + windows, images, heads, windows)
    g = torch.Generator(device="cuda").manual_seed(windows)
    q, k, v = (torch.randn(images * windows, heads, 49, 32, generator=g, device="cuda") for _ in range(3))
    rel = window_bias(table, idx).cuda()
    m = None if mask is None else mask.cuda()
    full = window_attn_mask(table.cuda(), idx.cuda(), images, m)
    assert torch.equal(K.window_attention(q, k, v, rel, m), K.qflash_forward(q, k, v, attn_mask=full))


@pytest.mark.gpu
def test_qwindowattention_module_equals_reference_formulation():
    from qflash_b200 import QWindowAttention
    torch.manual_seed(0)
    mod = QWindowAttention(dim=96, num_heads=3, window_size=7).cuda()
    x = torch.randn(32, 49, 96, device="cuda")
    mask = shifted_window_mask(28, 28, 7, 3).cuda()                      # 16 windows, 2 images
    out = mod(x, mask)
    # the reference module's own computation (qflash/attention.py:67-79)
    B_, N, C = x.shape
    qkv = mod.qkv(x).reshape(B_, N, 3, 3, -1).permute(2, 0, 3, 1, 4)
    q, k, v = qkv.unbind(0)
    am = mod._get_rel_pos_bias() + mask.view(1, 16, 1, N, N).expand(2, -1, 3, -1, -1).reshape(-1, 3, N, N)
    ref = mod.proj(K.qflash_forward(q, k, v, attn_mask=am).transpose(1, 2).reshape(B_, N, -1))
    assert torch.equal(out, ref)


def _swin_gpu_parts(heads, windows, images, dtype, table_dtype, mask_dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    N, D = 49, 32
    q, k, v = (torch.randn(images * windows, heads, N, D, generator=g, device="cuda").to(dtype) for _ in range(3))
    table = (torch.randn(169, heads, generator=g, device="cuda") * 2).to(table_dtype)
    index = relative_position_index(7, 7).cuda()
    side = int(windows ** 0.5) * 7
    mask = shifted_window_mask(side, side, 7, 3).cuda().to(mask_dtype) if windows > 1 else None
    return q, k, v, table, index, mask


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,table_dtype,mask_dtype", [
    (torch.float32, torch.float32, torch.float32),
    (torch.float16, torch.float16, torch.float16),
    (torch.bfloat16, torch.bfloat16, torch.bfloat16),
    (torch.float16, torch.float32, torch.float16),    # promoted add in fp32
    (torch.bfloat16, torch.float16, torch.bfloat16),  # fp16 + bf16 -> fp32
])
@pytest.mark.parametrize("windows", [1, 16])
def test_window_bias_built_on_device_equals_reference_mask(dtype, table_dtype, mask_dtype, windows):
    """qflash_fwd_fused_window (bias from table, index and mask on the device)
    equals qflash.forward on the dense [B_, H, N, N] mask QWindowAttention
    builds (qflash/attention.py:68-72), bit for bit."""
    heads, images = 3, 2
    q, k, v, table, index, mask = _swin_gpu_parts(heads, windows, images, dtype, table_dtype, mask_dtype)
    full = window_attn_mask(table, index, images * windows // (mask.shape[0] if mask is not None else 1)
                            if mask is not None else images, mask)
    expect = K.forward_with_scales(q, k, v, full)
    got = K.forward_window_fused(q, k, v, table, index, mask)
    assert torch.equal(got, expect)


@pytest.mark.gpu
def test_window_bias_bad_index_raises():
    q, k, v, table, index, mask = _swin_gpu_parts(3, 16, 1, torch.float16, torch.float16, torch.float16)
    bad = index.clone()
    bad[3, 5] = 169
    with pytest.raises(IndexError):
        K.forward_window_fused(q, k, v, table, bad, mask)
    assert torch.isnan(K.forward_window_fused(q, k, v, table, bad, mask, check=False)).all()


@pytest.mark.gpu
def test_qwindowattention_fused_equals_host_path(monkeypatch):
    from qflash_b200.attention import QWindowAttention
    torch.manual_seed(0)
    m = QWindowAttention(96, 3, 7).cuda().half()
    x = torch.randn(2 * 16, 49, 96, device="cuda", dtype=torch.half)
    mask = shifted_window_mask(28, 28, 7, 3).cuda().half()
    monkeypatch.setattr(K, "FUSED", False)
    ref = m(x, mask)
    ref_nomask = m(x)
    monkeypatch.setattr(K, "FUSED", True)
    assert torch.equal(m(x, mask), ref)
    assert torch.equal(m(x), ref_nomask)
