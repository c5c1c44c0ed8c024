"""SQNR of the public qflash.forward against scaled-dot-product attention on the
reference benchmark's own inputs (benchmark.py:17-28: torch.manual_seed(199),
then per workload torch.rand(3, Z, H, N, D) * 8 - 4 in fp16 on CUDA, followed by
the latency runs' draws at batch multipliers 1 and 8).  The figure must equal
the oracle's on the same int8 tensors within 0.01 dB.  The published A2 / A7
figures (README.md:27-30, 32.50 / 31.02 dB) were measured on another GPU: CUDA's
Philox stream depends on the launch grid, so after the first draw the seeded
inputs differ between GPUs, and A7 does not reproduce from the seed even on the
CPU generator (33.3 dB); the values measured here are printed beside them."""
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import qflash_oracle as orc

pytestmark = pytest.mark.gpu

# benchmark.py:6-15 (name, Z, H, N, D) and its batch multipliers
SHAPES = [("A1", 1, 3, 197, 64), ("A2", 1, 6, 197, 64), ("A3", 1, 12, 197, 64), ("A4", 64, 3, 49, 32),
          ("A5", 16, 6, 49, 32), ("A6", 4, 12, 49, 32), ("A7", 1, 24, 49, 32)]
BATCHES = [1, 8]
PUBLISHED = {"A2": 32.50, "A7": 31.02}


def _inputs(name):
    """q, k, v of workload `name` exactly as benchmark.py draws them."""
    torch.manual_seed(199)
    for nm, Z, H, N, D in SHAPES:
        qkv = torch.rand(3, Z, H, N, D, device="cuda", dtype=torch.float16) * 8 - 4
        if nm == name:
            return qkv[0], qkv[1], qkv[2]
        for b in BATCHES:                      # the latency runs' draws
            torch.rand(3, Z * b, H, N, D, device="cuda", dtype=torch.float16)
    raise KeyError(name)


def _sqnr(ref, out):
    # benchmark.py:28 on fp16 tensors: 20 log10(|ref| / |out - ref|)
    return float(20 * torch.log10(torch.norm(ref) / torch.norm(out - ref)))


@pytest.mark.parametrize("name", ["A2", "A7"])
def test_sqnr_matches_oracle_and_published(name):
    import qflash
    from qflash_b200 import kernel as K
    q, k, v = _inputs(name)
    out = qflash.qflash.forward(q, k, v)
    ref = F.scaled_dot_product_attention(q, k, v)
    s_ours = _sqnr(ref, out)
    qs, ks, vs = (t.abs().amax() / 127 for t in (q, k, v))
    sm, rs, eM, rM, lM, aM = K.fixed_point_params(float((qs * ks).item()), q.shape[-1], None)
    q8, k8, v8 = (K.quantize(t, s).cpu().numpy() for t, s in ((q, qs), (k, ks), (v, vs)))
    o_or = torch.from_numpy(orc.attention_int8(q8, k8, v8, orc.Params(sm, rs, eM, rM, lM, aM))).cuda() * vs
    s_or = _sqnr(ref, o_or)
    print(f"{name}: SQNR {s_ours:.2f} dB (oracle {s_or:.2f} dB, published {PUBLISHED[name]:.2f} dB on another GPU)")
    assert math.isfinite(s_ours) and abs(s_ours - s_or) <= 0.01, (s_ours, s_or)
