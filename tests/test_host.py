"""Host-side mirror of qflash/kernel.py:283-336 against the reference's captured launches (CPU)."""
import numpy as np
import pytest
import torch

from conftest import golden_cases
from qflash_b200 import kernel as K


def _scale(rec):
    s = float(rec["scale"])
    return None if np.isnan(s) else s


@pytest.mark.parametrize("name", golden_cases())
def test_fixed_point_params(golden, name):
    rec = golden(name)
    _, _, _, ls, as_ = (int(x) for x in rec["flags"])
    D = rec["q8"].shape[-1]
    _, rs, eM, rM, lM, aM = K.fixed_point_params(float(rec["qk_scale"]), D, _scale(rec), ls, as_)
    assert [rs, eM, rM, lM, aM] == rec["params"].tolist()


@pytest.mark.parametrize("name", golden_cases())
def test_quantize_and_scales(golden, name):
    rec = golden(name)
    q, k, v = (torch.from_numpy(rec[x]) for x in "qkv")
    qs = q.abs().amax() / 127
    ks = k.abs().amax() / 127
    vs = v.abs().amax() / 127
    assert float((qs * ks).item()) == float(rec["qk_scale"])
    assert float(vs) == float(rec["o_scale"])
    for t, s, ref in ((q, qs, "q8"), (k, ks, "k8"), (v, vs, "v8")):
        np.testing.assert_array_equal(K.quantize(t, s).numpy(), rec[ref])


@pytest.mark.parametrize("name", [n for n in golden_cases() if n.startswith(("bool", "float", "cfg4"))])
def test_quantize_bias_matches_reference_cpu(golden, name):
    rec = golden(name)
    mask = torch.from_numpy(rec["mask"])
    Z, H, N, _ = rec["q8"].shape
    sm_scale, *_ = K.fixed_point_params(float(rec["qk_scale"]), rec["q8"].shape[-1], _scale(rec))
    bias, strides = K.quantize_bias(mask, sm_scale, Z, H, N)
    assert strides[3] == 1 and strides[2] % 4 == 0
    full = torch.as_strided(bias, (Z, H, N, N), strides)
    np.testing.assert_array_equal(full.numpy(), rec["bias"])


def test_arith_flags():
    assert K.arith_flags(True, True, True, "full") == 0          # the reference as compiled on B200
    assert K.arith_flags(True, True, True, "ieee") == 16
    assert K.arith_flags(False, True, True, "ieee") == 1 | 16
    assert K.arith_flags(True, False, False, "full") == 2 | 4
    with pytest.raises(ValueError):
        K.arith_flags(div_mode="fast")


def test_head_dim_checks():
    x = torch.zeros(1, 1, 4, 16)
    with pytest.raises(ValueError):
        K.qflash_forward(x, x, x)
    with pytest.raises(AssertionError):
        K.qflash_forward(torch.zeros(1, 1, 4, 32), torch.zeros(1, 1, 4, 64), torch.zeros(1, 1, 4, 64))
    with pytest.raises(ValueError):  # CPU tensors: no CPU path
        K.qflash_forward(torch.ones(1, 1, 4, 32), torch.ones(1, 1, 4, 32), torch.ones(1, 1, 4, 32))


def test_public_surface():
    import qflash
    import qflash_b200
    assert qflash.qflash is qflash_b200.qflash
    assert callable(qflash.qflash.forward) and len(qflash.qflash.kernel) == 1
    for n in ("QAttention", "QWindowAttention", "patch_attention"):
        assert getattr(qflash, n) is getattr(qflash_b200, n)
