"""Swin window-attention helpers, written from their definitions.

``QWindowAttention`` (qflash/attention.py:39-86) takes its relative-position
index from timm (``get_relative_position_index``) and receives timm's
shifted-window mask.  timm is optional here, so both are defined below from
the Swin Transformer construction they follow.
"""
from __future__ import annotations

import torch


def relative_position_index(win_h: int, win_w: int) -> torch.Tensor:
    """Index [N, N] (N = win_h * win_w) into the (2*win_h-1)*(2*win_w-1)
    bias table: for query token i at (y_i, x_i) and key token j at (y_j, x_j),
    ((y_i - y_j) + win_h - 1) * (2*win_w - 1) + (x_i - x_j) + win_w - 1."""
    ys, xs = torch.meshgrid(torch.arange(win_h), torch.arange(win_w), indexing="ij")
    ys = ys.reshape(-1)
    xs = xs.reshape(-1)
    dy = ys[:, None] - ys[None, :] + (win_h - 1)
    dx = xs[:, None] - xs[None, :] + (win_w - 1)
    return (dy * (2 * win_w - 1) + dx).to(torch.long)


def shifted_window_mask(img_h: int, img_w: int, window: int, shift: int,
                        masked_value: float = -100.0) -> torch.Tensor:
    """Additive mask [nW, N, N] of a cyclically shifted window partition.

    After a cyclic shift by ``shift`` the image splits into 3 x 3 regions
    (row bands [0, H-window), [H-window, H-shift), [H-shift, H) and the same
    for columns).  Two tokens of one window may attend to each other only if
    they come from the same region; other pairs get ``masked_value``.
    Windows are numbered row-major over the (img_h/window) x (img_w/window)
    grid, tokens row-major inside a window.
    """
    label = torch.zeros(img_h, img_w, dtype=torch.long)
    bands_h = [(0, img_h - window), (img_h - window, img_h - shift), (img_h - shift, img_h)]
    bands_w = [(0, img_w - window), (img_w - window, img_w - shift), (img_w - shift, img_w)]
    region = 0
    for h0, h1 in bands_h:
        for w0, w1 in bands_w:
            label[h0:h1, w0:w1] = region
            region += 1
    nh, nw = img_h // window, img_w // window
    win = label.view(nh, window, nw, window).permute(0, 2, 1, 3).reshape(nh * nw, window * window)
    same = win[:, :, None] == win[:, None, :]
    mask = torch.zeros(nh * nw, window * window, window * window, dtype=torch.float32)
    mask.masked_fill_(~same, masked_value)
    return mask


def window_bias(table: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """Relative-position bias [1, H, N, N] gathered from ``table`` [T, H]
    (qflash/attention.py:58-61)."""
    n = index.shape[0]
    b = table[index.reshape(-1)].view(n, n, -1).permute(2, 0, 1).contiguous()
    return b.unsqueeze(0)


def window_attn_mask(table: torch.Tensor, index: torch.Tensor, num_images: int,
                     mask: torch.Tensor | None) -> torch.Tensor:
    """The float ``attn_mask`` that QWindowAttention.forward hands to
    ``qflash.forward`` (qflash/attention.py:68-74): bias + the window mask
    broadcast over images and heads, shape [B_, H, N, N] (or [1, H, N, N]
    without a mask)."""
    attn_mask = window_bias(table, index)
    if mask is None:
        return attn_mask
    nW, n, _ = mask.shape
    heads = table.shape[1]
    m = mask.view(1, nW, 1, n, n).expand(num_images, -1, heads, -1, -1)
    return attn_mask + m.reshape(-1, heads, n, n)
