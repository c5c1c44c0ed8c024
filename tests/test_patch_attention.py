"""patch_attention (qflash/attention.py:89-108) on CPU: timm is absent here, so
stand-in timm modules are registered in sys.modules; the swap logic -- which
submodules are replaced, that weights carry over, what is counted -- is what
this checks (the replaced modules' forward is covered by the GPU tests)."""
import sys
import types

import torch
from torch import nn


class _Attention(nn.Module):
    def __init__(self, dim, num_heads, qkv_bias=True):
        super().__init__()
        self.num_heads = num_heads
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)


class _WindowAttention(nn.Module):
    def __init__(self, dim, num_heads, window_size):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.window_size = (window_size, window_size)
        self.relative_position_bias_table = nn.Parameter(torch.randn((2 * window_size - 1) ** 2, num_heads))
        self.qkv = nn.Linear(dim, 3 * dim)
        self.proj = nn.Linear(dim, dim)


def _install_stub_timm(monkeypatch):
    timm = types.ModuleType("timm")
    layers = types.ModuleType("timm.layers")
    attention = types.ModuleType("timm.layers.attention")
    models = types.ModuleType("timm.models")
    swin = types.ModuleType("timm.models.swin_transformer")
    attention.Attention = _Attention
    swin.WindowAttention = _WindowAttention
    timm.layers, timm.models, layers.attention, models.swin_transformer = layers, models, attention, swin
    for name, mod in (("timm", timm), ("timm.layers", layers), ("timm.layers.attention", attention),
                      ("timm.models", models), ("timm.models.swin_transformer", swin)):
        monkeypatch.setitem(sys.modules, name, mod)


def test_patch_attention_swaps_timm_modules(monkeypatch):
    _install_stub_timm(monkeypatch)
    from qflash_b200.attention import QAttention, QWindowAttention, patch_attention
    torch.manual_seed(0)
    model = nn.Sequential(
        nn.ModuleDict({"attn": _Attention(64, 4), "mlp": nn.Linear(64, 64)}),
        nn.ModuleDict({"attn": _WindowAttention(96, 3, 7)}),
        _Attention(32, 2, qkv_bias=False),
    )
    before = {k: v.clone() for k, v in model.state_dict().items()}
    counts = patch_attention(model)
    assert counts == {"attn": 2, "wattn": 1}
    assert isinstance(model[0]["attn"], QAttention) and isinstance(model[2], QAttention)
    assert isinstance(model[1]["attn"], QWindowAttention)
    assert isinstance(model[0]["mlp"], nn.Linear)
    assert model[2].qkv.bias is None and model[0]["attn"].num_heads == 4
    after = model.state_dict()
    for k, v in before.items():            # every weight carries over unchanged
        assert torch.equal(after[k], v), k
    assert patch_attention(model) == {"attn": 0, "wattn": 0}   # nothing left to swap
