"""QAttention / QWindowAttention / patch_attention: the reference's model
integration (qflash/attention.py:12-108) over this package's qflash.forward.

timm is optional: its helpers are replaced by local equivalents when it is not
installed; ``patch_attention`` needs timm (it swaps timm modules).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
from torch import nn

from . import kernel as K
from .kernel import qflash, window_attention
from .swin import relative_position_index

try:  # pragma: no cover - exercised only where timm is installed
    from timm.layers import to_2tuple, trunc_normal_
    from timm.models.swin_transformer import get_relative_position_index
except ImportError:
    def to_2tuple(x):
        return tuple(x) if isinstance(x, (tuple, list)) else (x, x)

    def trunc_normal_(t, std=1.0):
        return nn.init.trunc_normal_(t, std=std)

    def get_relative_position_index(win_h, win_w):
        return relative_position_index(win_h, win_w)


class QAttention(nn.Module):
    """qflash/attention.py:12-36."""

    def __init__(self, dim: int, num_heads: int, qkv_bias: bool = True):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)

    def forward(self, x: torch.Tensor, attn_mask: Optional[torch.Tensor] = None,
                is_causal: bool = False) -> torch.Tensor:
        B, N, C = x.shape
        qkv = self.qkv(x).reshape(B, N, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        q, k, v = qkv.unbind(0)
        if K.FUSED and attn_mask is None and x.is_cuda:
            # the attention epilogue writes [B, N, H, D] directly: the reshape
            # below is then a view instead of a transpose copy
            out = torch.empty((B, N, self.num_heads, self.head_dim), dtype=q.dtype, device=x.device)
            # check: raise where the reference's qflash.forward raises (an all-zero q or k)
            K.forward_fused(q, k, v, out=out.permute(0, 2, 1, 3), check=True)
            return self.proj(out.reshape(B, N, C))
        x = qflash.forward(q, k, v, attn_mask=attn_mask)
        return self.proj(x.transpose(1, 2).reshape(B, N, C))

    @classmethod
    def from_orig(cls, src: nn.Module) -> "QAttention":
        new = cls(
            dim=src.qkv.in_features,
            num_heads=src.num_heads,
            qkv_bias=src.qkv.bias is not None,
        ).to(device=src.qkv.weight.device, dtype=src.qkv.weight.dtype)
        new.load_state_dict(src.state_dict())
        return new


class QWindowAttention(nn.Module):
    """qflash/attention.py:39-86."""

    def __init__(self, dim: int, num_heads: int, window_size, qkv_bias: bool = True):
        super().__init__()
        self.dim = dim
        self.num_heads = num_heads
        self.window_size = to_2tuple(window_size)
        win_h, win_w = self.window_size
        self.window_area = win_h * win_w
        self.relative_position_bias_table = nn.Parameter(
            torch.empty((2 * win_h - 1) * (2 * win_w - 1), num_heads))
        self.register_buffer(
            "relative_position_index",
            get_relative_position_index(win_h, win_w),
            persistent=False,
        )
        self.qkv = nn.Linear(dim, dim * 3, bias=qkv_bias)
        self.proj = nn.Linear(dim, dim)
        trunc_normal_(self.relative_position_bias_table, std=.02)

    def _get_rel_pos_bias(self) -> torch.Tensor:
        bias = self.relative_position_bias_table[self.relative_position_index.view(-1)]
        bias = bias.view(self.window_area, self.window_area, -1).permute(2, 0, 1).contiguous()
        return bias.unsqueeze(0)

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        B_, N, C = x.shape
        qkv = self.qkv(x).reshape(B_, N, 3, self.num_heads, -1).permute(2, 0, 3, 1, 4)
        q, k, v = qkv.unbind(0)

        # the reference adds the (window) mask to the bias at full batch size and
        # calls qflash.forward(q, k, v, attn_mask=...); the per-window forms below
        # give the same result (see their docstrings)
        if K.FUSED and x.is_cuda and q.dtype in (torch.float32, torch.float16, torch.bfloat16):
            # bias built on the device from table, index and mask; output written
            # in the [B_, N, H, D] layout the reshape below takes as a view
            out = torch.empty((B_, N, self.num_heads, q.shape[-1]), dtype=q.dtype, device=x.device)
            K.forward_window_fused(q, k, v, self.relative_position_bias_table, self.relative_position_index,
                                   mask, out=out.permute(0, 2, 1, 3))
            return self.proj(out.reshape(B_, N, -1))
        x = window_attention(q, k, v, self._get_rel_pos_bias(), mask)
        return self.proj(x.transpose(1, 2).reshape(B_, N, -1))

    @classmethod
    def from_orig(cls, src: nn.Module) -> "QWindowAttention":
        new = cls(
            dim=src.dim,
            num_heads=src.num_heads,
            window_size=src.window_size,
            qkv_bias=src.qkv.bias is not None,
        ).to(device=src.qkv.weight.device, dtype=src.qkv.weight.dtype)
        new.load_state_dict(src.state_dict())
        return new


def patch_attention(model: nn.Module) -> Dict[str, int]:
    """Replace every timm ``Attention`` / ``WindowAttention`` submodule of
    ``model`` by QAttention / QWindowAttention carrying the same weights
    (qflash/attention.py:89-108); returns how many of each were replaced.
    Needs timm."""
    import timm.layers.attention as timm_attention
    import timm.models.swin_transformer as timm_swin

    replacement = ((timm_attention.Attention, QAttention, "attn"),
                   (timm_swin.WindowAttention, QWindowAttention, "wattn"))
    # decide on the original tree first, then swap (named_modules would walk the new modules)
    plan = []
    for name, module in model.named_modules():
        for timm_cls, q_cls, key in replacement:
            if isinstance(module, timm_cls):
                plan.append((name, q_cls, key))
                break
    counts = {"attn": 0, "wattn": 0}
    for name, q_cls, key in plan:
        owner_name, _, attr = name.rpartition(".")
        owner = model.get_submodule(owner_name) if owner_name else model
        setattr(owner, attr, q_cls.from_orig(getattr(owner, attr)))
        counts[key] += 1
    return counts
