"""sm_100a kernel (through the C ABI) against the reference's outputs: bit-exact int8."""
import numpy as np
import pytest
import torch

from conftest import golden_cases
from oracle import qflash_oracle as orc

pytestmark = pytest.mark.gpu


def _run_kernel(rec, flags=None):
    from qflash_b200 import kernel as K
    q8, k8, v8 = (torch.from_numpy(rec[x]).cuda() for x in ("q8", "k8", "v8"))
    o8 = torch.empty_like(v8)
    rs, eM, rM, lM, aM = (int(x) for x in rec["params"])
    e, l, a, ls, as_ = (int(x) for x in rec["flags"])
    if flags is None:
        flags = K.arith_flags(bool(e), bool(l), bool(a), "ieee")
    bias = bs = None
    if "bias" in rec:
        b = torch.from_numpy(rec["bias"]).cuda()
        Z, H, N, _ = b.shape
        N4 = (N + 3) // 4 * 4
        bias = torch.zeros((Z, H, N, N4), dtype=torch.int32, device="cuda")
        bias[..., :N] = b
        bs = list(bias.stride())
    K.launch_int8(q8, k8, v8, o8, rs, eM, rM, lM, aM, bias, bs, ls, as_, flags)
    torch.cuda.synchronize()
    return o8.cpu().numpy()


@pytest.mark.parametrize("name", golden_cases())
def test_kernel_matches_reference(golden, name):
    rec = golden(name)
    o = _run_kernel(rec)
    mism = int((o != rec["o8"]).sum())
    assert mism == 0, f"{mism} of {o.size} int8 outputs differ"


@pytest.mark.parametrize("rpi", ["32", "64", "128"])
@pytest.mark.parametrize("name", ["cfg1_vit_s", "cfg5_vit_l", "n129_d64", "n100_d32", "n65_d32", "n197_d128",
                                  "n80_d256", "env_exp_idiv", "env_acc_idiv", "env_shift40", "bool_mask",
                                  "expm_check_1100", "expm_wrap"])
def test_rows_per_item_forced(golden, name, rpi, monkeypatch):
    """Work items of 32, 64 and 128 query rows (chosen by grid size unless
    QFLASH_ROWS_PER_ITEM forces one) give the same bit-exact output."""
    monkeypatch.setenv("QFLASH_ROWS_PER_ITEM", rpi)
    rec = golden(name)
    o = _run_kernel(rec)
    mism = int((o != rec["o8"]).sum())
    assert mism == 0, f"{mism} of {o.size} int8 outputs differ"


def _triton_gpu(name):
    with np.load(__import__("conftest").GOLDEN / "triton_gpu" / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.mark.parametrize("name", ["cfg1_vit_s", "cfg2_vit_b", "cfg3_deit_t", "cfg5_vit_l", "bench_a2_fp16",
                                  "bench_a7_fp16", "n80_d256", "n197_d128", "strided_qattn", "bool_mask",
                                  "bool_mask_full_row", "float_mask_m100", "cfg4_swin_s1", "cfg4_swin_s4"])
def test_forward_end_to_end(golden, name):
    """The public qflash.forward (on-device path, default final division) on the
    float inputs returns exactly what the reference's compiled Triton kernel
    returns on B200: o8 * o_scale with o8 from tests/golden/triton_gpu (for the
    masked cases the bias is built on the device, as the reference builds it
    on CUDA)."""
    import qflash
    rec = golden(name)
    gpu = _triton_gpu(name)
    q, k, v = (torch.from_numpy(rec[x]).cuda() for x in "qkv")
    mask = torch.from_numpy(rec["mask"]).cuda() if "mask" in rec else None
    s = float(rec["scale"])
    out = qflash.qflash.forward(q, k, v, attn_mask=mask, scale=None if np.isnan(s) else s)
    assert out.dtype == q.dtype and out.shape == q.shape
    o_scale = v.abs().amax() / 127
    expect = torch.from_numpy(gpu["o8"]).cuda() * o_scale
    mism = int((out != expect).sum())
    assert mism == 0, f"{mism} of {out.numel()} outputs differ from the compiled reference"


@pytest.mark.parametrize("name", ["cfg1_vit_s", "bench_a2_fp16", "bool_mask", "cfg4_swin_s1"])
def test_forward_host_path_end_to_end(golden, name, monkeypatch):
    """The torch-op host path of qflash.forward (QFLASH_FUSED=0) gives the same."""
    import qflash
    from qflash_b200 import kernel as K
    monkeypatch.setattr(K, "FUSED", False)
    rec = golden(name)
    gpu = _triton_gpu(name)
    q, k, v = (torch.from_numpy(rec[x]).cuda() for x in "qkv")
    mask = torch.from_numpy(rec["mask"]).cuda() if "mask" in rec else None
    s = float(rec["scale"])
    out = qflash.qflash.forward(q, k, v, attn_mask=mask, scale=None if np.isnan(s) else s)
    expect = torch.from_numpy(gpu["o8"]).cuda() * (v.abs().amax() / 127)
    assert torch.equal(out, expect)


def test_device_error_word_clear():
    from qflash_b200 import _lib
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0


TRITON_GPU = sorted(p.stem for p in (__import__("conftest").GOLDEN / "triton_gpu").glob("*.npz"))


@pytest.mark.parametrize("explicit", [False, True])
@pytest.mark.parametrize("name", TRITON_GPU)
def test_default_division_matches_compiled_reference_on_b200(golden, name, explicit):
    """The default final division (flags 0, or QFLASH_FLAG_DIV_FULL given
    explicitly) reproduces the reference's compiled Triton kernel on B200
    (approximate fp32 divide), captured by tests/golden/gen_golden_triton_gpu.py."""
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    rec = dict(golden(name))
    gpu = _triton_gpu(name)
    if "bias" in gpu:
        rec["bias"] = gpu["bias"]          # the GPU host path's bias (reciprocal-multiply rounding)
    e, l, a, _, _ = (int(x) for x in rec["flags"])
    flags = K.arith_flags(bool(e), bool(l), bool(a), "full") | (_lib.FLAG_DIV_FULL if explicit else 0)
    o = _run_kernel(rec, flags=flags)
    mism = int((o != gpu["o8"]).sum())
    assert mism == 0, f"{mism} of {o.size} int8 outputs differ from the compiled reference"


@pytest.mark.parametrize("rpi", ["32", "64"])
@pytest.mark.parametrize("name", ["cfg2_vit_b", "cfg5_vit_l", "bool_mask", "n65_d32"])
def test_default_division_small_items(golden, name, rpi, monkeypatch):
    """Same, with the small work items that small grids use."""
    from qflash_b200 import kernel as K
    monkeypatch.setenv("QFLASH_ROWS_PER_ITEM", rpi)
    rec = dict(golden(name))
    gpu = _triton_gpu(name)
    if "bias" in gpu:
        rec["bias"] = gpu["bias"]
    e, l, a, _, _ = (int(x) for x in rec["flags"])
    o = _run_kernel(rec, flags=K.arith_flags(bool(e), bool(l), bool(a), "full"))
    assert int((o != gpu["o8"]).sum()) == 0


def test_conflicting_division_flags_rejected():
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    x = torch.zeros(1, 1, 32, 32, dtype=torch.int8, device="cuda")
    with pytest.raises(RuntimeError, match="exclusive"):
        K.launch_int8(x, x, x, torch.empty_like(x), 4033, -16, 2064, 266239, 266239,
                      flags=_lib.FLAG_DIV_FULL | _lib.FLAG_DIV_IEEE)


def test_bounded_wait_reports_timeout_and_context_stays_usable():
    """A wait on an mbarrier that nothing arrives at gives up after its cycle
    limit and records the error bit instead of hanging; the context then runs
    the attention kernel normally."""
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    stream = torch.cuda.current_stream().cuda_stream
    assert _lib.device_error(stream) == 0
    assert _lib.load().qflash_selftest_wait_timeout(stream, 2_000_000) == 0   # ~1 ms at 1.9 GHz
    assert _lib.device_error(stream) == 1 << 31
    assert _lib.device_error(stream) == 0                                     # read-and-clear
    q, k, v = (torch.randn(1, 2, 64, 64, device="cuda") for _ in range(3))
    assert torch.equal(K.forward_fused(q, k, v), K.forward_with_scales(q, k, v))
    assert _lib.device_error(stream) == 0


@pytest.mark.parametrize("N,D", [(49, 32), (96, 64), (65, 64), (33, 32), (130, 32)])
def test_many_heads_of_few_chunks(N, D):
    """Launches with many work items of one to five 32-key chunks each (the
    Swin window shape among them) run every pipeline stage many times round;
    a sample of heads is compared with the oracle bit for bit and the bounded
    waits must report nothing."""
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    g = torch.Generator().manual_seed(N * 1000 + D)
    Z, H = 400, 3
    q, k, v = (torch.randn(Z, H, N, D, generator=g) for _ in range(3))
    qs, ks, vs = (t.abs().amax() / 127 for t in (q, k, v))
    sm, rs, eM, rM, lM, aM = K.fixed_point_params(float(qs * ks), D, None)
    q8, k8, v8 = (K.quantize(t, s) for t, s in ((q, qs), (k, ks), (v, vs)))
    d8 = [t.cuda() for t in (q8, k8, v8)]
    o8 = torch.empty_like(d8[2])
    stream = torch.cuda.current_stream().cuda_stream
    K.launch_int8(*d8, o8, rs, eM, rM, lM, aM, flags=K.arith_flags(div_mode="ieee"))
    torch.cuda.synchronize()
    assert _lib.device_error(stream) == 0
    sel = torch.randperm(Z * H, generator=g)[:12]
    zs, hs = (sel // H).numpy(), (sel % H).numpy()
    prm = orc.Params(sm, rs, eM, rM, lM, aM)
    got = o8.cpu().numpy()
    for z, h in zip(zs, hs):
        ref = orc.attention_int8(q8[z:z + 1, h:h + 1].numpy(), k8[z:z + 1, h:h + 1].numpy(),
                                 v8[z:z + 1, h:h + 1].numpy(), prm)
        assert np.array_equal(ref[0, 0], got[z, h]), f"head ({z}, {h}) differs"


def _oracle_head(args):
    q, k, v, prm = args
    return orc.attention_int8(q, k, v, prm)[0, 0]


def test_full_vit_b_workload_every_head():
    """The whole ViT-B attention layer (3072 heads, many work items per CTA, the
    second 128-row tile of each head partly past N) against the oracle on every
    head (IEEE division, as the oracle computes): catches anything that depends
    on the order of items within a CTA (e.g. TMEM reuse between items)."""
    import multiprocessing as mp
    import os
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    from qflash_b200.workloads import WORKLOADS, make_inputs
    w = WORKLOADS["vit_b"]
    q, k, v, _ = make_inputs(w, seed=11, device="cuda")
    qs, ks, vs = (t.abs().amax() / 127 for t in (q, k, v))
    sm, rs, eM, rM, lM, aM = K.fixed_point_params(float((qs * ks).item()), w.D, None)
    q8, k8, v8 = K.quantize(q, qs), K.quantize(k, ks), K.quantize(v, vs)
    o8 = torch.empty_like(v8)
    for _ in range(3):   # repeated launches: timing-dependent faults get several chances
        K.launch_int8(q8, k8, v8, o8, rs, eM, rM, lM, aM, flags=K.arith_flags(div_mode="ieee"))
        torch.cuda.synchronize()
        assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
        got = o8.cpu().numpy()
        prm = orc.Params(sm, rs, eM, rM, lM, aM)
        q8n, k8n, v8n = (t.cpu().numpy() for t in (q8, k8, v8))
        tasks = [(q8n[z:z + 1, h:h + 1], k8n[z:z + 1, h:h + 1], v8n[z:z + 1, h:h + 1], prm)
                 for z in range(w.Z) for h in range(w.H)]
        with mp.get_context("spawn").Pool(max(1, min(32, os.cpu_count() or 1))) as pool:
            refs = pool.map(_oracle_head, tasks, chunksize=64)
        bad = [(i // w.H, i % w.H) for i, r in enumerate(refs) if not np.array_equal(r, got[i // w.H, i % w.H])]
        assert not bad, f"{len(bad)} heads differ, e.g. {bad[:5]}"
