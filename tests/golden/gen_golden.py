"""Generate the golden vectors in tests/golden/ from the reference itself.

Runs the reference's own Triton kernels (EfficientCompLab/qflash,
qflash/kernel.py) on CPU under TRITON_INTERPRET=1 and records, for each case,
the float inputs, the host-derived fixed-point parameters, the int8 tensors and
int32 bias the kernel was launched with, the int8 output it wrote and the
dequantised result ``qflash.forward`` returned.

Only this script reads the reference (its checkout root given by --ref or
the QFLASH_REFERENCE_ROOT environment variable).  It must run where the reference
and Triton are available; the .npz files it writes are committed and are all
the tests need.

    python tests/golden/gen_golden.py [--ref /path/to/qflash] [--only NAME]
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
import time
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from qflash_b200.swin import relative_position_index, shifted_window_mask, window_attn_mask  # noqa: E402

FLAG_ENV = ("QFLASH_EXP_USE_SHIFT", "QFLASH_L_USE_SHIFT", "QFLASH_ACC_USE_SHIFT",
            "QFLASH_L_SHIFT", "QFLASH_ACC_SHIFT")


def load_reference(ref_root: str, env: dict[str, str], tag: str):
    """Import qflash/kernel.py by path (its package __init__ needs timm) with
    the QFLASH_* environment it reads at import time."""
    saved = {k: os.environ.get(k) for k in FLAG_ENV}
    for k in FLAG_ENV:
        os.environ.pop(k, None)
    os.environ.update(env)
    try:
        spec = importlib.util.spec_from_file_location(f"qflash_ref_{tag}", os.path.join(ref_root, "qflash", "kernel.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return mod


class Spy:
    """Stands in for a Triton kernel object: records the launch arguments."""

    def __init__(self, kern):
        self.kern = kern
        self.calls = []

    def __getitem__(self, grid):
        def launch(*args, **kw):
            self.kern[grid](*args, **kw)
            self.calls.append((args, kw))
        return launch


def run_case(mod, q, k, v, attn_mask=None, scale=None):
    """Call the reference forward and capture its kernel launch."""
    spy_u, spy_m = Spy(mod.qflash_kernel), Spy(mod.qflash_masked_kernel)
    orig = (mod.qflash_kernel, mod.qflash_masked_kernel)
    mod.qflash_kernel, mod.qflash_masked_kernel = spy_u, spy_m
    try:
        out = mod.qflash.forward(q, k, v, attn_mask=attn_mask, scale=scale)
    finally:
        mod.qflash_kernel, mod.qflash_masked_kernel = orig
    (args, kw), = spy_u.calls + spy_m.calls
    masked = bool(spy_m.calls)
    q8, k8, v8, o8 = args[:4]
    rest = args[5:] if masked else args[4:]
    params = [int(x) for x in rest[:5]]
    rec = dict(q8=q8.numpy(), k8=k8.numpy(), v8=v8.numpy(), o8=o8.numpy(),
               params=np.array(params, dtype=np.int64),
               flags=np.array([int(kw["EXP_USE_SHIFT"]), int(kw["L_USE_SHIFT"]), int(kw["ACC_USE_SHIFT"]),
                               kw["L_SHIFT"], kw["ACC_SHIFT"]], dtype=np.int64),
               q_strides=np.array(q8.stride(), dtype=np.int64))
    if masked:
        rec["bias"] = args[4].numpy()
    # forward returned o * o_scale; keep o_scale (as float64) and check that identity
    o_scale = v.abs().amax() / 127
    assert torch.equal(out, o8 * o_scale)
    rec["o_scale"] = np.array(float(o_scale))
    rec["qk_scale"] = np.array(float((q.abs().amax() / 127 * (k.abs().amax() / 127)).item()))
    return rec


def gen(seed, shape, kind="normal", dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    if kind == "normal":
        xs = [torch.randn(shape, generator=g) for _ in range(3)]
    elif kind == "uniform4":        # benchmark.py:136 distribution
        xs = [torch.rand(shape, generator=g) * 8 - 4 for _ in range(3)]
    elif kind == "head_std":
        xs = [torch.randn(shape, generator=g) * (torch.rand((1, shape[1], 1, 1), generator=g) * 1.5 + 0.5)
              for _ in range(3)]
    elif kind == "outlier":
        xs = []
        for _ in range(3):
            x = torch.randn(shape, generator=g)
            sel = torch.rand(shape, generator=g) < 0.01
            xs.append(torch.where(sel, x * 8, x))
    else:
        raise ValueError(kind)
    return [x.to(dtype) for x in xs]


def swin_mask(seed, images, heads, windows):
    g = torch.Generator().manual_seed(seed + 1000)
    table = torch.randn((169, heads), generator=g) * 0.02
    idx = relative_position_index(7, 7)
    mask = None
    if windows > 1:
        side = int(round(windows ** 0.5)) * 7
        mask = shifted_window_mask(side, side, 7, 3)
    return window_attn_mask(table, idx, images, mask)


def cases():
    """(name, env, builder) -- builder returns (q, k, v, attn_mask, scale)."""
    D = {}
    # the ViT-S/B/L, DeiT-T and Swin-T workloads at reduced batch (same N, d, H-distribution)
    D["cfg1_vit_s"] = ({}, lambda: (*gen(1, (1, 3, 197, 64)), None, None))
    D["cfg2_vit_b"] = ({}, lambda: (*gen(2, (1, 4, 197, 64), "head_std"), None, None))
    D["cfg3_deit_t"] = ({}, lambda: (*gen(3, (1, 3, 197, 64), "outlier"), None, None))
    D["cfg4_swin_s1"] = ({}, lambda: (*gen(4, (8, 3, 49, 32)), swin_mask(4, 2, 3, 4), None))
    D["cfg4_swin_s4"] = ({}, lambda: (*gen(5, (1, 24, 49, 32)), swin_mask(5, 1, 24, 1), None))
    D["cfg5_vit_l"] = ({}, lambda: (*gen(6, (1, 2, 577, 64)), None, None))
    # benchmark.py workload shapes / distribution (fp16, U(-4, 4))
    D["bench_a2_fp16"] = ({}, lambda: (*gen(7, (1, 6, 197, 64), "uniform4", torch.float16), None, None))
    D["bench_a7_fp16"] = ({}, lambda: (*gen(8, (1, 24, 49, 32), "uniform4", torch.float16), None, None))
    # ragged / tiny sequence lengths and other head dims
    for n in (1, 7, 31, 32, 33, 64, 65, 100):
        D[f"n{n}_d32"] = ({}, lambda n=n: (*gen(100 + n, (1, 2, n, 32)), None, None))
    D["n129_d64"] = ({}, lambda: (*gen(11, (1, 2, 129, 64)), None, None))
    D["n197_d128"] = ({}, lambda: (*gen(12, (1, 2, 197, 128)), None, None))
    D["n80_d256"] = ({}, lambda: (*gen(13, (1, 1, 80, 256)), None, None))
    # scale extremes: requant of the row max wraps past 127, exp_M large (int32 wrap of x*exp_M)
    D["wrap_scale200"] = ({}, lambda: (*gen(14, (1, 2, 197, 64)), None, 200.0))
    D["wrap_scale40"] = ({}, lambda: (*gen(15, (1, 2, 197, 64)), None, 40.0))
    D["expm_wrap"] = ({}, lambda: (*gen(16, (1, 2, 197, 64), "outlier"), None, 2.0))
    D["tiny_scale"] = ({}, lambda: (*gen(17, (1, 2, 100, 64)), None, 0.01))

    def tuned(seed, shape, kind, exp_m):
        """inputs plus the `scale` argument that puts exp_M near -exp_m"""
        q, k, v = gen(seed, shape, kind)
        qk = float((q.abs().amax() / 127 * (k.abs().amax() / 127)).item())
        return q, k, v, None, (exp_m / 65536.0) / (1.44269504 * qk)
    D["expm_check_1100"] = ({}, lambda: tuned(31, (1, 3, 197, 64), "outlier", 1100))
    D["expm_check_d128"] = ({}, lambda: tuned(32, (1, 2, 130, 128), "normal", 600))
    # masks
    def boolmask():
        q, k, v = gen(18, (2, 2, 70, 32))
        g = torch.Generator().manual_seed(19)
        m = torch.rand((2, 1, 70, 70), generator=g) > 0.3
        m[..., 0] = True
        return q, k, v, m, None
    D["bool_mask"] = ({}, boolmask)
    def floatmask():
        q, k, v = gen(20, (1, 2, 60, 32))
        g = torch.Generator().manual_seed(21)
        m = torch.randn((1, 2, 60, 60), generator=g)
        sel = torch.rand((1, 2, 60, 60), generator=g)
        m = torch.where(sel < 0.2, torch.full_like(m, -100.0), m)   # exactly -100: not masked
        m = torch.where(sel > 0.9, torch.full_like(m, -150.0), m)   # < -100: masked
        return q, k, v, m, None
    D["float_mask_m100"] = ({}, floatmask)
    def allmasked_row():
        q, k, v = gen(22, (1, 1, 40, 32))
        m = torch.ones((1, 1, 40, 40), dtype=torch.bool)
        m[0, 0, 3, :] = False          # a fully masked query row
        return q, k, v, m, None
    D["bool_mask_full_row"] = ({}, allmasked_row)
    # non-contiguous strides (QAttention layout: qkv -> (3, B, H, N, D) permute)
    def strided():
        g = torch.Generator().manual_seed(23)
        qkv = torch.randn(2, 50, 3, 3, 32, generator=g).permute(2, 0, 3, 1, 4)
        return qkv[0], qkv[1], qkv[2], None, None
    D["strided_qattn"] = ({}, strided)
    # alternative arithmetic selected by QFLASH_* environment flags
    D["env_exp_idiv"] = ({"QFLASH_EXP_USE_SHIFT": "0"}, lambda: (*gen(24, (1, 2, 197, 64)), None, None))
    D["env_l_idiv"] = ({"QFLASH_L_USE_SHIFT": "0"}, lambda: (*gen(25, (1, 2, 100, 64)), None, None))
    D["env_acc_idiv"] = ({"QFLASH_ACC_USE_SHIFT": "0"}, lambda: (*gen(26, (1, 2, 100, 64)), None, None))
    D["env_all_idiv"] = ({"QFLASH_EXP_USE_SHIFT": "0", "QFLASH_L_USE_SHIFT": "0", "QFLASH_ACC_USE_SHIFT": "0"},
                         lambda: (*gen(27, (1, 2, 49, 32)), None, None))
    D["env_shift20_24"] = ({"QFLASH_L_SHIFT": "20", "QFLASH_ACC_SHIFT": "24"},
                           lambda: (*gen(28, (1, 2, 197, 64)), None, None))
    D["env_shift40"] = ({"QFLASH_L_SHIFT": "40", "QFLASH_ACC_SHIFT": "40"},
                        lambda: (*gen(29, (1, 2, 100, 64)), None, None))
    return D


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("QFLASH_REFERENCE_ROOT"),
                    required="QFLASH_REFERENCE_ROOT" not in os.environ,
                    help="root of the reference checkout (or set QFLASH_REFERENCE_ROOT)")
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    mods = {}
    for name, (env, build) in cases().items():
        if a.only and a.only != name:
            continue
        key = tuple(sorted(env.items()))
        if key not in mods:
            mods[key] = load_reference(a.ref, env, f"m{len(mods)}")
        q, k, v, mask, scale = build()
        t0 = time.time()
        rec = run_case(mods[key], q, k, v, mask, scale)
        rec.update(q=q.numpy(), k=k.numpy(), v=v.numpy(),
                   in_dtype=np.array(str(q.dtype)), scale=np.array(np.nan if scale is None else scale),
                   env=np.array(repr(sorted(env.items()))))
        if mask is not None:
            rec["mask"] = mask.numpy()
        np.savez_compressed(HERE / f"{name}.npz", **rec)
        print(f"{name:22s} {tuple(q.shape)} params={rec['params'].tolist()} {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
