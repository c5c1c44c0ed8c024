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


@pytest.mark.parametrize("name", ["cfg1_vit_s", "cfg3_deit_t", "bench_a2_fp16", "n80_d256"])
def test_forward_end_to_end(golden, name):
    """qflash.forward on the float inputs: same int8 output, same returned values."""
    import qflash
    rec = golden(name)
    q, k, v = (torch.from_numpy(rec[x]).cuda() for x in "qkv")
    mask = torch.from_numpy(rec["mask"]).cuda() if "mask" in rec else None
    s = float(rec["scale"])
    out = qflash.qflash.forward(q, k, v, attn_mask=mask, scale=None if np.isnan(s) else s)
    assert out.dtype == q.dtype and out.shape == q.shape
    o_scale = v.abs().amax() / 127
    expect = torch.from_numpy(rec["o8"]).cuda() * o_scale
    assert torch.equal(out, expect)


def test_device_error_word_clear():
    from qflash_b200 import _lib
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0


TRITON_GPU = sorted(p.stem for p in (__import__("conftest").GOLDEN / "triton_gpu").glob("*.npz"))


@pytest.mark.parametrize("name", TRITON_GPU)
def test_div_full_matches_compiled_reference_on_b200(golden, name):
    """QFLASH_DIV=full reproduces the reference's compiled Triton kernel on B200
    (approximate fp32 divide), captured by tests/golden/gen_golden_triton_gpu.py."""
    import numpy as np
    from qflash_b200 import kernel as K
    rec = dict(golden(name))
    with np.load(__import__("conftest").GOLDEN / "triton_gpu" / f"{name}.npz") as z:
        gpu = {k: z[k] for k in z.files}
    if "bias" in gpu:
        rec["bias"] = gpu["bias"]          # the GPU host path's bias (reciprocal-multiply rounding)
    e, l, a, _, _ = (int(x) for x in rec["flags"])
    o = _run_kernel(rec, flags=K.arith_flags(bool(e), bool(l), bool(a), "full"))
    mism = int((o != gpu["o8"]).sum())
    assert mism == 0, f"{mism} of {o.size} int8 outputs differ from the compiled reference"
