"""CPU restatement of QFlash's integer-only attention forward (numpy).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``qflash_b200``)
imports this module; it is the checker that the sm_100a kernels are compared
against in ``tests/``, in ``__graft_entry__.smoke()`` and in the
``cpu_baseline`` leg of ``bench.py``.

Every function restates one piece of the reference implementation
(EfficientCompLab/qflash, ``qflash/kernel.py``) with the exact integer
semantics of that code:

* int32 arithmetic wraps modulo 2**32 (numpy int32 arrays wrap silently);
* ``>>`` on signed values is arithmetic, and a shift amount outside [0, 31]
  (negative, or >= 32) yields the sign fill 0 / -1 -- this is what the
  reference's interpreter run (numpy ``right_shift``) and the PTX ``shr.s32``
  clamp both produce;
* ``.to(int8)`` keeps the low 8 bits (128 -> -128);
* integer ``//`` truncates toward zero (Triton ``arith.divsi``);
* ``int / int`` is an IEEE fp32 division of the two values converted to fp32,
  then ``.to(int32)`` truncates toward zero; a NaN or out-of-range quotient
  becomes INT32_MIN (what the reference run on x86 numpy produces).

Parity pin: ``tests/golden/`` holds input/output vectors captured from the
reference's own Triton kernels (run on CPU under ``TRITON_INTERPRET=1`` by
``tests/golden/gen_golden.py``); ``tests/test_oracle_golden.py`` checks this
module bit for bit against every one of them.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

# qflash/kernel.py:137,288 -- the masking sentinel
NEG_INF = -(1 << 20)
# qflash/kernel.py:287
LOG2E = 1.44269504
# qflash/kernel.py:301 -- fixed-point bits of exp_M / req_M
SHIFT = 16
# every autotune config of the reference uses BLOCK_N = 32 (kernel.py:14-16,27);
# the chunked online softmax makes this width part of the arithmetic.
BLOCK_N = 32

INT32_MIN = -(1 << 31)


@dataclass(frozen=True)
class Params:
    """Fixed-point constants derived on the host (qflash/kernel.py:290-307)."""

    sm_scale: float
    sm_rscale: int
    exp_M: int
    req_M: int
    l_M: int
    acc_M: int
    l_shift: int = 30
    acc_shift: int = 30


def derive_params(qk_scale: float, head_dim: int, scale: float | None = None,
                  l_shift: int = 30, acc_shift: int = 30) -> Params:
    """qflash/kernel.py:290-307, in Python doubles exactly as the reference.

    ``qk_scale`` is ``(q_scale * k_scale).item()`` -- the product taken in the
    input dtype on the device, then widened to a Python float.
    """
    if scale is None:
        scale = 1.0 / (head_dim ** 0.5)
    scale = scale * LOG2E
    sm_scale = scale * qk_scale
    sm_rscale = int(round(1.0 / sm_scale))
    exp_M = int(round(-sm_scale * (1 << SHIFT)))
    req_M = int(round(sm_scale * 127 * (1 << SHIFT)))
    l_M = int(round((1 << l_shift) / sm_rscale))
    acc_M = int(round((1 << acc_shift) / sm_rscale))
    return Params(sm_scale, sm_rscale, exp_M, req_M, l_M, acc_M, l_shift, acc_shift)


# ---------------------------------------------------------------------------
# integer primitives
# ---------------------------------------------------------------------------

def _i32(x) -> np.ndarray:
    return np.asarray(x).astype(np.int32)


def sra32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Arithmetic right shift of int32 ``a`` by int32 ``b``; any shift amount
    outside [0, 31] gives the sign fill (0 or -1)."""
    a = _i32(a)
    b = np.asarray(b).astype(np.int64)
    ok = (b >= 0) & (b < 32)
    bs = np.where(ok, b, 31)
    return np.where(ok, a >> bs, a >> 31).astype(np.int32)


def trunc_div(a: np.ndarray, b) -> np.ndarray:
    """Integer division rounding toward zero (C / Triton semantics)."""
    a = np.asarray(a).astype(np.int64)
    b = np.asarray(b).astype(np.int64)
    q = np.abs(a) // np.abs(b)
    return np.where((a < 0) != (b < 0), -q, q)


def exp2_i32_shift(x: np.ndarray, rscale: int, exp_M: int) -> np.ndarray:
    """qflash/kernel.py:40-44: ~ rscale * 2**(x * sm_scale) for x <= 0."""
    x = _i32(x)
    q = (x * np.int32(exp_M)) >> SHIFT                       # int32 product wraps
    r = x + q * np.int32(rscale)                              # wraps
    return sra32((r >> 1) + np.int32(rscale), q)


def exp2_i32_idiv(x: np.ndarray, rscale: int) -> np.ndarray:
    """qflash/kernel.py:47-51 (QFLASH_EXP_USE_SHIFT=0)."""
    x = _i32(x)
    q = _i32(trunc_div(_i32(-x), rscale))                     # -x in int32 first
    r = x + q * np.int32(rscale)
    return sra32((r >> 1) + np.int32(rscale), q)


def exp2_i32(x, rscale, exp_M, use_shift=True):
    """qflash/kernel.py:54-59."""
    return exp2_i32_shift(x, rscale, exp_M) if use_shift else exp2_i32_idiv(x, rscale)


def requantize(p: np.ndarray, req_M: int) -> np.ndarray:
    """qflash/kernel.py:62-64: int8((p * req_M + 2**15) >> 16), wrapping."""
    p = _i32(p)
    return ((p * np.int32(req_M) + np.int32(1 << (SHIFT - 1))) >> SHIFT).astype(np.int8)


def scale_release_shift(x: np.ndarray, alpha: np.ndarray, M: int, shift: int) -> np.ndarray:
    """qflash/kernel.py:67-69: int32(((int64)x * alpha * M + 2**(S-1)) >> S)."""
    x = np.asarray(x).astype(np.int64)
    alpha = np.asarray(alpha).astype(np.int64)
    v = x * alpha * np.int64(M) + np.int64(1 << (shift - 1))
    return (v >> shift).astype(np.int32)


def scale_release_idiv(x: np.ndarray, alpha: np.ndarray, rscale: int) -> np.ndarray:
    """qflash/kernel.py:72-74: (x * alpha) // rscale with an int32 product."""
    prod = _i32(x) * _i32(alpha)                              # int32, wraps
    return _i32(trunc_div(prod, rscale))


def scale_release(x, alpha, rscale, M, shift, use_shift=True):
    """qflash/kernel.py:77-82."""
    if use_shift:
        return scale_release_shift(x, alpha, M, shift)
    return scale_release_idiv(x, alpha, rscale)


def div_to_int8(acc: np.ndarray, l: np.ndarray) -> np.ndarray:
    """qflash/kernel.py:176-178: int8(int32(fp32(acc) / fp32(l)))."""
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        qf = acc.astype(np.float32) / l.astype(np.float32)
    ok = (qf >= np.float32(-2147483648.0)) & (qf < np.float32(2147483648.0))
    qi = np.where(ok, np.where(ok, qf, 0).astype(np.float64).astype(np.int64), INT32_MIN)
    return qi.astype(np.int32).astype(np.int8)


# ---------------------------------------------------------------------------
# the fused forward
# ---------------------------------------------------------------------------

def attention_int8(q8, k8, v8, p: Params, bias=None, exp_use_shift=True,
                   l_use_shift=True, acc_use_shift=True, return_state=False):
    """Integer attention forward of qflash_kernel / qflash_masked_kernel.

    Follows qflash/kernel.py:137-180 (unmasked) and :240-272 (masked): one
    query row at a time (rows are independent), key/value chunks of
    ``BLOCK_N`` = 32 columns in order, integer online softmax between them.

    q8, k8, v8: int8 arrays [Z, H, N, D] (any strides).  bias: int32
    [Z, H, N, N] (or broadcastable) or None.  Returns int8 O [Z, H, N, D];
    with ``return_state`` also the final int32 ``acc`` and ``l``.
    """
    q8 = np.asarray(q8)
    Z, H, N, D = q8.shape
    ZH = Z * H
    q = q8.reshape(ZH, N, D).astype(np.int32)
    k = np.asarray(k8).reshape(ZH, N, D).astype(np.int32)
    v = np.asarray(v8).reshape(ZH, N, D).astype(np.int32)
    if bias is not None:
        bias = np.broadcast_to(np.asarray(bias), (Z, H, N, N)).reshape(ZH, N, N).astype(np.int32)

    rs, eM, rM = p.sm_rscale, p.exp_M, p.req_M
    m_i = np.full((ZH, N), NEG_INF, dtype=np.int32)
    l_i = np.ones((ZH, N), dtype=np.int32)
    acc = np.zeros((ZH, N, D), dtype=np.int32)

    for start in range(0, N, BLOCK_N):
        nc = min(BLOCK_N, N - start)
        kc = k[:, start:start + nc, :]
        s = np.matmul(q, kc.transpose(0, 2, 1))               # [ZH, N, nc] int32
        if bias is not None:
            s = s + bias[:, :, start:start + nc]              # int32 add, wraps
        if nc < BLOCK_N:                                       # out-of-range columns
            pad = np.full((ZH, N, BLOCK_N - nc), NEG_INF, dtype=np.int32)
            s = np.concatenate([s, pad], axis=2)
        m_ij = np.maximum(m_i, s.max(axis=2))
        x = s - m_ij[:, :, None]
        pe = exp2_i32(x, rs, eM, exp_use_shift)
        p8 = requantize(pe, rM)
        l_ij = p8.astype(np.int32).sum(axis=2, dtype=np.int32)
        alpha = exp2_i32(m_i - m_ij, rs, eM, exp_use_shift)
        l_i = scale_release(l_i, alpha, rs, p.l_M, p.l_shift, l_use_shift) + l_ij
        acc = scale_release(acc, alpha[:, :, None], rs, p.acc_M, p.acc_shift, acc_use_shift)
        vc = v[:, start:start + nc, :]
        acc = acc + np.matmul(p8[:, :, :nc].astype(np.int32), vc)
        m_i = m_ij

    o = div_to_int8(acc, l_i[:, :, None]).reshape(Z, H, N, D)
    if return_state:
        return o, acc.reshape(Z, H, N, D), l_i.reshape(Z, H, N)
    return o


# ---------------------------------------------------------------------------
# host-side float -> int helpers (reference performs these with torch ops)
# ---------------------------------------------------------------------------

def quantize_bias_float(attn_mask: np.ndarray, sm_scale: float, reciprocal: bool) -> np.ndarray:
    """qflash/kernel.py:333-336 for a float mask, in fp32.

    ``reciprocal`` selects torch's CUDA evaluation of ``x / python_scalar``
    (multiply by the fp32 reciprocal); False is the CPU true division.
    """
    a = np.asarray(attn_mask, dtype=np.float32)
    is_masked = a < np.float32(-1e2)
    clipped = np.where(is_masked, np.float32(0), a).astype(np.float32)
    t = (clipped * np.float32(LOG2E)).astype(np.float32)
    if reciprocal:
        t = (t * (np.float32(1.0) / np.float32(sm_scale))).astype(np.float32)
    else:
        t = (t / np.float32(sm_scale)).astype(np.float32)
    quant = np.rint(t).astype(np.int32)
    return np.where(is_masked, np.int32(NEG_INF), quant).astype(np.int32)


def quantize_bias_bool(attn_mask: np.ndarray) -> np.ndarray:
    """qflash/kernel.py:328-330: 0 where True, NEG_INF where False."""
    return np.where(np.asarray(attn_mask, dtype=bool), 0, NEG_INF).astype(np.int32)


def exact_quotients(q8, k8, v8, p: Params, bias=None, **flags) -> np.ndarray:
    """Boolean [Z, H, N, D]: where acc / l is an exact nonzero integer.

    These are the only elements where the reference's compiled GPU kernel
    (whose ``acc / l`` at qflash/kernel.py:176 is the approximate fp32 divide
    div.full.f32, at most 2 ulp from the quotient) can truncate differently
    from the IEEE division ``div_to_int8`` restates: while |acc| < 2^21 every
    other quotient is at least 1/l > 2.5 ulp away from an integer.  There it
    can land one below the integer, i.e. one step toward zero."""
    _, acc, l = attention_int8(q8, k8, v8, p, bias, return_state=True, **flags)
    l = l[..., None].astype(np.int64)
    acc = acc.astype(np.int64)
    return (acc != 0) & (l > 0) & (acc % np.maximum(l, 1) == 0)


def sqnr_db(ref: np.ndarray, out: np.ndarray) -> float:
    """benchmark.py:28 -- 20 log10(|ref| / |out - ref|)."""
    ref = np.asarray(ref, dtype=np.float64)
    out = np.asarray(out, dtype=np.float64)
    return float(20.0 * math.log10(np.linalg.norm(ref) / np.linalg.norm(out - ref)))
