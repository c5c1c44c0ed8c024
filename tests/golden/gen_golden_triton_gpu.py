"""Capture the reference's compiled Triton kernels on a B200 for every golden case.

Needs a GPU and the reference installed under baseline/_ref (pip --target).
For each tests/golden/<name>.npz it calls the reference ``qflash.forward`` on
the same float inputs on the GPU, captures the int8 kernel inputs and output
(as gen_golden.py does for the interpreted run) and writes
tests/golden/triton_gpu/<name>.npz (or --out DIR) with the GPU int8 output and, for masked
cases, the int32 bias the GPU host path produced (torch's CUDA division by a
Python scalar multiplies by a reciprocal, so it can differ from the CPU run).

    python tests/golden/gen_golden_triton_gpu.py [--ref baseline/_ref] [--out DIR]
"""
from __future__ import annotations

import os

# the compiled kernels, not the interpreter: Triton reads this when the module is imported
os.environ.pop("TRITON_INTERPRET", None)

import argparse
import glob
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
FLAG_ENV = ("QFLASH_EXP_USE_SHIFT", "QFLASH_L_USE_SHIFT", "QFLASH_ACC_USE_SHIFT",
            "QFLASH_L_SHIFT", "QFLASH_ACC_SHIFT")


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


def load(ref_root, env, tag):
    for k in FLAG_ENV:
        os.environ.pop(k, None)
    os.environ.update(env)
    spec = importlib.util.spec_from_file_location(f"qflash_gpu_{tag}", os.path.join(ref_root, "qflash", "kernel.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=str(HERE.parents[1] / "baseline" / "_ref"))
    ap.add_argument("--out", default=str(HERE / "triton_gpu"))
    a = ap.parse_args()
    assert os.environ.get("TRITON_INTERPRET", "0") != "1"
    out_dir = Path(a.out)
    out_dir.mkdir(exist_ok=True)
    mods = {}
    for path in sorted(glob.glob(str(HERE / "*.npz"))):
        name = Path(path).stem
        z = dict(np.load(path))
        env = dict(eval(str(z["env"])))
        key = repr(sorted(env.items()))
        if key not in mods:
            mods[key] = load(a.ref, env, str(len(mods)))
        m = mods[key]
        su, sm = Spy(m.qflash_kernel), Spy(m.qflash_masked_kernel)
        orig = (m.qflash_kernel, m.qflash_masked_kernel)
        m.qflash_kernel, m.qflash_masked_kernel = su, sm
        try:
            q, k, v = (torch.from_numpy(z[x]).cuda() for x in "qkv")
            mask = torch.from_numpy(z["mask"]).cuda() if "mask" in z else None
            s = float(z["scale"])
            m.qflash.forward(q, k, v, attn_mask=mask, scale=None if np.isnan(s) else s)
            torch.cuda.synchronize()
        finally:
            m.qflash_kernel, m.qflash_masked_kernel = orig
        (args, kw), = su.calls + sm.calls
        rec = {"o8": args[3].cpu().numpy()}
        for i, nm in enumerate(("q8", "k8", "v8")):
            assert np.array_equal(args[i].cpu().numpy(), z[nm]), (name, nm)
        if sm.calls:
            rec["bias"] = args[4].cpu().numpy()
        np.savez_compressed(out_dir / f"{name}.npz", **rec)
        d = int((rec["o8"] != z["o8"]).sum())
        print(f"{name:22s} differs from the interpreted run in {d} of {rec['o8'].size}", flush=True)


if __name__ == "__main__":
    main()
