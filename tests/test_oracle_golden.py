"""The numpy oracle against the reference's own outputs (tests/golden/)."""
import numpy as np
import pytest

from conftest import golden_cases
from oracle import qflash_oracle as orc


def _params(rec):
    rs, eM, rM, lM, aM = (int(x) for x in rec["params"])
    _, _, _, ls, as_ = (int(x) for x in rec["flags"])
    return orc.Params(float("nan"), rs, eM, rM, lM, aM, ls, as_)


@pytest.mark.parametrize("name", golden_cases())
def test_oracle_matches_reference_kernel(golden, name):
    rec = golden(name)
    e, l, a = (bool(x) for x in rec["flags"][:3])
    o = orc.attention_int8(rec["q8"], rec["k8"], rec["v8"], _params(rec), rec.get("bias"),
                           exp_use_shift=e, l_use_shift=l, acc_use_shift=a)
    assert o.dtype == np.int8
    np.testing.assert_array_equal(o, rec["o8"])
