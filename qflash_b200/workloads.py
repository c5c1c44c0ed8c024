"""Seeded synthetic attention inputs with the shapes and value distributions of
the benchmark configurations (ViT-S/B/L, DeiT-T, Swin-T stages 1 and 4).

The reference measures accuracy on ImageNet with pretrained timm models; no
dataset or weights are available here, so these generators stand in for the
attention-layer inputs of those models.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .swin import relative_position_index, shifted_window_mask, window_attn_mask, window_bias


@dataclass(frozen=True)
class Workload:
    name: str
    Z: int          # batch, or images x windows for Swin
    H: int
    N: int
    D: int
    dist: str       # "normal" | "head_std" | "outlier" | "swin"
    images: int = 0     # Swin: number of images (Z = images * windows)
    windows: int = 0    # Swin: windows per image (1 = no shift mask)

    @property
    def ops(self) -> int:
        """Algorithmic integer ops of one call: two GEMMs, 2*N*N*D MACs each."""
        return 4 * self.Z * self.H * self.N * self.N * self.D

    @property
    def io_bytes(self) -> int:
        """Algorithmic HBM bytes of one call: int8 Q, K, V read and O written."""
        return 4 * self.Z * self.H * self.N * self.D

    def scaled(self, Z: int) -> "Workload":
        if self.dist == "swin":
            images = max(1, Z // self.windows)
            return Workload(self.name, images * self.windows, self.H, self.N, self.D,
                            self.dist, images, self.windows)
        return Workload(self.name, Z, self.H, self.N, self.D, self.dist)


# ViT-S (the CPU case), ViT-B/16 (headline), DeiT-T, Swin-T stages 1 and 4, ViT-L/16 @384.
WORKLOADS = {
    "vit_s": Workload("vit_s", 8, 6, 197, 64, "normal"),
    "vit_b": Workload("vit_b", 256, 12, 197, 64, "head_std"),
    "deit_t": Workload("deit_t", 1024, 3, 197, 64, "outlier"),
    "swin_s1": Workload("swin_s1", 64 * 64, 3, 49, 32, "swin", images=64, windows=64),
    "swin_s4": Workload("swin_s4", 64, 24, 49, 32, "swin", images=64, windows=1),
    "vit_l": Workload("vit_l", 1024, 16, 577, 64, "normal"),
}


def _normal(shape, g, device, dtype):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dtype)


def make_inputs(w: Workload, seed: int = 0, device="cpu", dtype=torch.float32, parts: bool = False):
    """Return (q, k, v, attn_mask) for workload ``w``; attn_mask is None
    except for Swin, where it is the float bias(+shift mask) tensor that
    QWindowAttention builds at full batch size.  With ``parts`` a fifth item
    (rel_bias [1, H, N, N], window_mask [nW, N, N] or None) is appended (None
    for non-Swin workloads)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    shape = (w.Z, w.H, w.N, w.D)
    if w.dist in ("normal", "swin"):
        q, k, v = (_normal(shape, g, device, torch.float32) for _ in range(3))
    elif w.dist == "head_std":
        out = []
        for _ in range(3):
            std = torch.rand((1, w.H, 1, 1), generator=g, device=device) * 1.5 + 0.5
            out.append(_normal(shape, g, device, torch.float32) * std)
        q, k, v = out
    elif w.dist == "outlier":
        out = []
        for _ in range(3):
            x = _normal(shape, g, device, torch.float32)
            sel = torch.rand(shape, generator=g, device=device) < 0.01
            out.append(torch.where(sel, x * 8.0, x))
        q, k, v = out
    else:
        raise ValueError(w.dist)
    attn_mask = None
    win_parts = None
    if w.dist == "swin":
        win = 7
        table = torch.randn(((2 * win - 1) ** 2, w.H), generator=g, device=device) * 0.02
        index = relative_position_index(win, win).to(device)
        mask = None
        if w.windows > 1:
            side = int(round(w.windows ** 0.5)) * win
            mask = shifted_window_mask(side, side, win, win // 2).to(device)
        attn_mask = window_attn_mask(table, index, w.images, mask)
        win_parts = (window_bias(table, index), mask)
    out = (q.to(dtype), k.to(dtype), v.to(dtype), attn_mask)
    return out + (win_parts,) if parts else out
