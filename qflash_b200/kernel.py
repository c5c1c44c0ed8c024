"""``qflash.forward``: QFlash's integer-only attention forward on B200.

Host side of the drop-in replacement for qflash/kernel.py:275-356.  The host
math (scale derivation, fixed-point constants in Python doubles, per-tensor
int8 quantisation, bias quantisation) follows the reference step for step so
that the int8 tensors and constants the kernel receives are bit-identical;
the two Triton launches are replaced by one call into the C ABI
(``qflash_i8_fwd``, include/qflash_b200.h) whose sm_100a kernel computes the
same int8 output.

Environment flags, read once at import like the reference (kernel.py:30-36):
QFLASH_EXP_USE_SHIFT, QFLASH_L_USE_SHIFT, QFLASH_ACC_USE_SHIFT (default 1),
QFLASH_L_SHIFT, QFLASH_ACC_SHIFT (default 30).  QFLASH_AUTOTUNE and
QFLASH_CUDA_GRAPH are accepted; they only pick Triton launch configurations
there and change no arithmetic, and this kernel has a single configuration.
QFLASH_DIV selects the rounding of the final fp32 division acc / l
(kernel.py:176): "full" (default; the approximate fp32 divide div.full.f32 that
the reference's compiled Triton kernel uses on B200, so the output is bit for
bit what the reference produces there) or "ieee" (IEEE round-to-nearest, as the
reference's interpreted run computes it).  QFLASH_FUSED=1 routes qflash.forward
(output mode) through ``forward_fused``: the same result without the host
synchronisation; inputs for which the reference raises (all-zero q or k)
then give an all-NaN output instead of an exception.
"""
from __future__ import annotations

import os

import torch
from torch import Tensor

from . import _lib

AUTOTUNE_SETTING = os.environ.get("QFLASH_AUTOTUNE", "default")
USE_CUDA_GRAPH = os.environ.get("QFLASH_CUDA_GRAPH", "0") == "1"
EXP_USE_SHIFT = os.environ.get("QFLASH_EXP_USE_SHIFT", "1") == "1"
L_USE_SHIFT = os.environ.get("QFLASH_L_USE_SHIFT", "1") == "1"
ACC_USE_SHIFT = os.environ.get("QFLASH_ACC_USE_SHIFT", "1") == "1"
L_SHIFT = int(os.environ.get("QFLASH_L_SHIFT", "30"))
ACC_SHIFT = int(os.environ.get("QFLASH_ACC_SHIFT", "30"))
DIV_MODE = os.environ.get("QFLASH_DIV", "full")
# qflash.forward runs every step on the device (forward_fused) unless
# QFLASH_FUSED=0 selects the torch-op host path (the reference's own sequence)
FUSED = os.environ.get("QFLASH_FUSED", "1") == "1"

LOG2E = 1.44269504
NEG_INF = -(1 << 20)
SHIFT = 16


def arith_flags(exp_use_shift=None, l_use_shift=None, acc_use_shift=None, div_mode=None) -> int:
    """C-ABI flag word for the QFLASH_* arithmetic switches."""
    f = 0
    if not (EXP_USE_SHIFT if exp_use_shift is None else exp_use_shift):
        f |= _lib.FLAG_EXP_IDIV
    if not (L_USE_SHIFT if l_use_shift is None else l_use_shift):
        f |= _lib.FLAG_L_IDIV
    if not (ACC_USE_SHIFT if acc_use_shift is None else acc_use_shift):
        f |= _lib.FLAG_ACC_IDIV
    mode = DIV_MODE if div_mode is None else div_mode
    if mode not in ("ieee", "full"):
        raise ValueError(f"QFLASH_DIV must be 'ieee' or 'full', got {mode!r}")
    if mode == "ieee":
        f |= _lib.FLAG_DIV_IEEE
    return f


def fixed_point_params(qk_scale: float, head_dim: int, scale: float | None,
                       l_shift: int = None, acc_shift: int = None):
    """qflash/kernel.py:290-307 in Python doubles: returns
    (sm_scale, sm_rscale, exp_M, req_M, l_M, acc_M)."""
    l_shift = L_SHIFT if l_shift is None else l_shift
    acc_shift = ACC_SHIFT if acc_shift is None else acc_shift
    if scale is None:
        scale = 1.0 / (head_dim ** 0.5)
    scale = scale * LOG2E
    sm_scale = scale * qk_scale
    sm_rscale = int(round(1.0 / sm_scale))
    exp_M = int(round(-sm_scale * (1 << SHIFT)))
    req_M = int(round(sm_scale * 127 * (1 << SHIFT)))
    l_M = int(round((1 << l_shift) / sm_rscale))
    acc_M = int(round((1 << acc_shift) / sm_rscale))
    return sm_scale, sm_rscale, exp_M, req_M, l_M, acc_M


def quantize(x: Tensor, s: Tensor) -> Tensor:
    """qflash/kernel.py:309-311: int8(clamp(round(x / s), -128, 127))."""
    return torch.clamp(torch.round(x / s), -128, 127).to(torch.int8)


def quantize_bias(attn_mask: Tensor, sm_scale: float, Z: int, H: int, N: int):
    """qflash/kernel.py:328-336 without the .expand().contiguous() copy.

    The same torch ops run on the mask at its own (broadcastable) shape --
    elementwise ops commute with broadcasting, so every value equals the
    reference's -- and the result is laid out as [Zb, Hb, N, N4] int32 with
    the row pitch N4 padded to a multiple of 4 (16 bytes, a TMA requirement).
    Returns (bias, element strides with 0 on broadcast dimensions).
    """
    if attn_mask.dtype == torch.bool:
        bias = torch.where(attn_mask, 0, NEG_INF).to(torch.int32)
    else:
        is_masked = attn_mask < -1e2
        clipped = attn_mask.masked_fill(is_masked, 0.0)
        quant = (clipped * LOG2E / sm_scale).round().to(torch.int32)
        bias = quant.masked_fill(is_masked, NEG_INF)
    while bias.dim() < 4:
        bias = bias.unsqueeze(0)
    if bias.dim() != 4:
        raise ValueError(f"attn_mask must broadcast to (Z, H, N, N); got shape {tuple(attn_mask.shape)}")
    Zb = Z if bias.shape[0] != 1 else 1
    Hb = H if bias.shape[1] != 1 else 1
    bias = bias.expand(Zb, Hb, N, N)
    N4 = (N + 3) // 4 * 4
    out = torch.empty((Zb, Hb, N, N4), dtype=torch.int32, device=bias.device)
    out[..., :N].copy_(bias)
    st = out.stride()
    return out, [st[0] if Zb > 1 else 0, st[1] if Hb > 1 else 0, st[2], 1]


def do_bench(fn, warmup: float = 10, rep: float = 100) -> float:
    """Median kernel time in ms: warm-up and repetition budgets in ms, the L2
    flushed (256 MB written) before every timed run, CUDA events around each
    run -- the method of the reference's latency mode (kernel.py:348-349)."""
    fn()
    torch.cuda.synchronize()
    cache = torch.empty(int(256e6 // 4), dtype=torch.int32, device="cuda")
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(5):
        cache.zero_()
        fn()
    e.record()
    torch.cuda.synchronize()
    est = s.elapsed_time(e) / 5
    n_warm = max(1, int(warmup / est))
    n_rep = max(1, int(rep / est))
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_rep)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_rep)]
    for _ in range(n_warm):
        fn()
    for i in range(n_rep):
        cache.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    times = sorted(a.elapsed_time(b) for a, b in zip(starts, ends))
    return times[len(times) // 2] if len(times) % 2 else 0.5 * (times[len(times) // 2 - 1] + times[len(times) // 2])


def launch_int8(q8: Tensor, k8: Tensor, v8: Tensor, o8: Tensor, sm_rscale: int, exp_M: int, req_M: int,
                l_M: int, acc_M: int, bias: Tensor | None = None, bias_strides=None,
                l_shift: int = None, acc_shift: int = None, flags: int = None, stream=None,
                bias_z_period: int = 0, o_peers=None, barrier=None) -> None:
    """Run the sm_100a kernel on int8 [Z, H, N, D] tensors already on the GPU
    (the launch at qflash/kernel.py:319-326 / 339-346).  ``o_peers``: addresses
    of o8's rows in other GPUs' copies of a gathered output (``shard.PeerOutput``),
    which the epilogue fills as well; ``barrier``: the gather barrier's
    (sig, sig_peers, rank, epoch), after which the kernel completes only once
    every rank's rows are in every copy."""
    for t in (q8, k8, v8, o8):
        if not t.is_cuda or t.dtype != torch.int8 or t.dim() != 4:
            raise ValueError("q, k, v, o must be 4-D int8 CUDA tensors")
    Z, H, N, D = q8.shape
    if stream is None:
        stream = torch.cuda.current_stream(q8.device).cuda_stream
    for name, val in (("exp_M", exp_M), ("req_M", req_M), ("sm_rscale", sm_rscale)):
        if not -(1 << 31) <= val < (1 << 31):
            raise OverflowError(f"{name}={val} does not fit in int32")
    _lib.i8_fwd(q8, k8, v8, o8, bias, bias_strides, Z, H, N, D, sm_rscale, exp_M, req_M, l_M, acc_M,
                L_SHIFT if l_shift is None else l_shift, ACC_SHIFT if acc_shift is None else acc_shift,
                arith_flags() if flags is None else flags, stream, bias_z_period, o_peers, barrier)


def qflash_forward(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    attn_mask: Tensor | None = None,
    scale: float | None = None,
    return_mode: str = 'output',
):
    """Integer-only attention; same signature, arithmetic and output dtype as
    the reference's ``qflash.forward`` (qflash/kernel.py:275-351).

    By default the whole forward runs on the device (``forward_fused``, bit for
    bit the same output) with one synchronisation at the end that raises where
    the reference raises (ZeroDivisionError for an all-zero q or k; ValueError
    when the constants are not representable).  Inputs it does not take (other
    dtypes, q/k/v of different shapes, masks that do not broadcast per batch
    and head) and ``return_mode='latency'`` use the torch-op host path."""
    if FUSED and return_mode == 'output' and _fused_takes(query, key, value, attn_mask):
        return forward_fused(query, key, value, attn_mask, scale, check=True)
    return forward_with_scales(query, key, value, attn_mask, scale, return_mode)


def _fused_takes(query, key, value, attn_mask) -> bool:
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        return False
    if query.dtype not in (torch.float32, torch.float16, torch.bfloat16) or not (
            query.dtype == key.dtype == value.dtype):
        return False
    if query.dim() != 4 or not (query.shape == key.shape == value.shape) or query.shape[-1] not in (32, 64, 128, 256):
        return False
    if attn_mask is not None:
        if not attn_mask.is_cuda or attn_mask.dtype not in (torch.float32, torch.float16, torch.bfloat16, torch.bool):
            return False
        m = attn_mask
        while m.dim() < 4:
            m = m.unsqueeze(0)
        Z, H, N, _ = query.shape
        if m.dim() != 4 or m.shape[0] not in (1, Z) or m.shape[1] not in (1, H) or m.shape[2] not in (1, N) \
                or m.shape[3] not in (1, N):
            return False
    return True


def forward_fused(query, key, value, attn_mask=None, scale=None, bias_z_period=0, check=False,
                  return_int8=False, return_workspace=False, out=None):
    """``qflash.forward`` with every step on the device (``qflash_fwd_fused``):
    no ``.item()`` synchronisation, no torch quantisation passes.  The output
    equals ``qflash.forward``'s bit for bit (contiguous [Z, H, N, D], input
    dtype).  ``check`` synchronises and raises where the reference raises
    (ZeroDivisionError for an all-zero q or k); without it such inputs give
    an all-NaN output.  ``bias_z_period`` as in ``forward_with_scales``.

    Unless ``return_int8`` is set, the attention epilogue writes the
    dequantised output itself (``qflash_fwd_fused_out``): into ``out`` when
    given (a [Z, H, N, D] tensor or view of the input dtype with a contiguous
    head dim, e.g. a permuted [Z, N, H, D] buffer), else into a new contiguous
    tensor."""
    D = query.shape[-1]
    assert query.shape[-1] == key.shape[-1] == value.shape[-1]
    assert D in {16, 32, 64, 128, 256}
    if D == 16:
        raise ValueError("head dim 16 is not supported (the chunk width 32 exceeds it), as in the reference")
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise ValueError("qflash.forward runs on CUDA tensors only")
    if not (query.dim() == 4 and query.shape == key.shape == value.shape):
        raise ValueError(f"fused path takes q, k, v of one [Z, H, N, D] shape, got "
                         f"{tuple(query.shape)}, {tuple(key.shape)}, {tuple(value.shape)}")
    if query.dtype not in (torch.float32, torch.float16, torch.bfloat16) or not (
            query.dtype == key.dtype == value.dtype):
        raise ValueError(f"fused path takes float32/float16/bfloat16 inputs of one dtype, got {query.dtype}")
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (query, key, value))
    Z, H, N, _ = q.shape
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    mask, mstr, zb, hb = None, None, 0, 0
    if attn_mask is not None:
        m = attn_mask
        while m.dim() < 4:
            m = m.unsqueeze(0)
        zb, hb = m.shape[0], m.shape[1]
        if zb not in (1, Z, bias_z_period) or hb not in (1, H):
            raise ValueError(f"attn_mask of shape {tuple(attn_mask.shape)} does not broadcast to {(Z, H, N, N)}")
        m = m.expand(zb, hb, N, N)
        mask = m
        mstr = [0 if m.shape[i] == 1 else m.stride(i) for i in range(4)]
    dev = q.device
    q8, k8, v8 = torch.empty((3, Z, H, N, D), dtype=torch.int8, device=dev).unbind(0)  # one allocation
    if out is None:
        out = torch.empty((Z, H, N, D), dtype=q.dtype, device=dev)
    elif out.shape != (Z, H, N, D) or out.dtype != q.dtype or out.stride(-1) != 1 or out.device != dev:
        raise ValueError(f"out must be a {(Z, H, N, D)} {q.dtype} tensor on {dev} with a contiguous last dim")
    ws = torch.empty(_lib.fused_workspace_bytes(zb, hb, N), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    period = bias_z_period if mask is not None else 0
    if return_int8:
        if not out.is_contiguous():
            raise ValueError("return_int8 needs a contiguous output")
        o8 = torch.empty((Z, H, N, D), dtype=torch.int8, device=dev)
        _lib.fwd_fused(q, k, v, mask, mstr, zb, hb, period, q8, k8, v8, o8, out,
                       scale * LOG2E, L_SHIFT, ACC_SHIFT, arith_flags(), ws, stream)
    else:
        _lib.fwd_fused_out(q, k, v, mask, mstr, zb, hb, period, q8, k8, v8, out,
                           scale * LOG2E, L_SHIFT, ACC_SHIFT, arith_flags(), ws, stream)
    if check:
        st = _lib.fused_status(ws, stream)
        if st == 1:
            raise ZeroDivisionError("float division by zero (q or k is all zero)")
        if st != 0:
            raise ValueError("the fixed-point constants are not representable for this input")
    extra = []
    if return_int8:
        extra.append((q8, k8, v8, o8))
    if return_workspace:
        extra.append(ws)
    return (out, *extra) if extra else out


def tensor_scales(query: Tensor, key: Tensor, value: Tensor):
    """qflash/kernel.py:294-296: per-tensor symmetric scales amax/127, in the
    input dtype."""
    i8max = torch.iinfo(torch.int8).max
    return query.abs().amax() / i8max, key.abs().amax() / i8max, value.abs().amax() / i8max


def forward_with_scales(query, key, value, attn_mask=None, scale=None, return_mode='output',
                        scales=None, launch=None, return_int8=False, bias_z_period=0,
                        o_out=None, o_peers=None, dequant=True, barrier=None):
    """The body of ``qflash.forward`` with seams: ``scales`` supplies
    (q_scale, k_scale, o_scale) computed elsewhere (the sharded path reduces
    them over all ranks so each shard quantises exactly like the whole
    tensor), ``launch`` replaces the kernel launch (host-logic tests), and
    ``return_int8`` also returns (o8, o_scale); ``bias_z_period`` > 0 means
    ``attn_mask`` has that many batch entries and batch z uses entry
    z % bias_z_period (see ``window_attention``).  ``o_out`` is the int8 output
    tensor to write (default: a new one), ``o_peers`` the addresses of its rows
    in other GPUs' copies (``shard.PeerOutput``), ``barrier`` the gather
    barrier of that launch, and ``dequant=False`` skips the local
    ``o * o_scale`` (returned as None)."""
    HEAD_DIM_Q, HEAD_DIM_K = query.shape[-1], key.shape[-1]
    HEAD_DIM_V = value.shape[-1]
    assert HEAD_DIM_Q == HEAD_DIM_K and HEAD_DIM_K == HEAD_DIM_V
    assert HEAD_DIM_K in {16, 32, 64, 128, 256}
    if HEAD_DIM_K == 16:
        # the reference fails to compile here: tl.static_assert(BLOCK_N <= HEAD_DIM), BLOCK_N = 32
        raise ValueError("head dim 16 is not supported (the chunk width 32 exceeds it), as in the reference")
    if launch is None and not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise ValueError("qflash.forward runs on CUDA tensors only")

    q_scale, k_scale, o_scale = tensor_scales(query, key, value) if scales is None else scales
    qk_scale = (q_scale * k_scale).item()
    sm_scale, sm_rscale, exp_M, req_M, l_M, acc_M = fixed_point_params(qk_scale, HEAD_DIM_Q, scale)

    query = quantize(query, q_scale)
    key = quantize(key, k_scale)
    value = quantize(value, o_scale)
    # the TMA loads need the head dim innermost (the reference takes any strides)
    query, key, value = (t if t.stride(-1) == 1 else t.contiguous() for t in (query, key, value))
    if o_out is None:
        o = torch.empty_like(value)
    else:
        if o_out.dtype != torch.int8 or o_out.shape != value.shape or o_out.stride(-1) != 1:
            raise ValueError(f"o_out must be int8 {tuple(value.shape)} with the head dim contiguous")
        o = o_out

    Z, H, N = query.shape[0], query.shape[1], query.shape[2]
    bias, bias_strides = None, None
    if attn_mask is not None:
        bias, bias_strides = quantize_bias(attn_mask, sm_scale, bias_z_period or Z, H, N)

    def kernel():
        if launch is not None:
            launch(query, key, value, o, sm_rscale, exp_M, req_M, l_M, acc_M, bias, bias_strides)
        else:
            launch_int8(query, key, value, o, sm_rscale, exp_M, req_M, l_M, acc_M, bias, bias_strides,
                        bias_z_period=bias_z_period, o_peers=o_peers, barrier=barrier)

    if return_mode == 'latency':
        return do_bench(kernel, warmup=10, rep=100)
    kernel()
    out = o * o_scale if dequant else None
    if return_int8:
        return out, o, o_scale
    return out


def forward_window_fused(query, key, value, table, index, window_mask=None, scale=None, check=True, out=None):
    """QWindowAttention's attention (qflash/attention.py:63-75) with every step
    on the device, the bias included (qflash_fwd_fused_window): the float mask
    entry (b, h, i, j) is table[index[i, j], h] + window_mask[b % nW, i, j],
    formed and quantised once per window and head.  Same bits as
    ``qflash.forward(q, k, v, attn_mask=<the reference's expanded mask>)``.

    table: [(2wh-1)(2ww-1), H]; index: [N, N] int64; window_mask: [nW, N, N] or
    None; q/k/v: [B_, H, N, D] with B_ a multiple of nW."""
    Z, H, N, D = query.shape
    if not (query.shape == key.shape == value.shape) or D not in (32, 64, 128, 256):
        raise ValueError("q, k, v must share one [B_, H, N, D] shape with D in {32, 64, 128, 256}")
    if query.dtype not in (torch.float32, torch.float16, torch.bfloat16) or not (
            query.dtype == key.dtype == value.dtype):
        raise ValueError(f"float32/float16/bfloat16 inputs of one dtype, got {query.dtype}")
    if table.dim() != 2 or table.shape[1] != H or index.numel() != N * N:
        raise ValueError(f"table must be [T, {H}] and index [{N}, {N}]")
    if scale is None:
        scale = 1.0 / (D ** 0.5)
    q, k, v = (t if t.stride(-1) == 1 else t.contiguous() for t in (query, key, value))
    dev = q.device
    idx = index.to(device=dev, dtype=torch.int64).contiguous().view(-1)
    tab = table.to(dev)
    nW = 0
    wm = None
    if window_mask is not None:
        wm = window_mask.to(dev).contiguous()
        nW = wm.shape[0]
        if wm.shape != (nW, N, N) or Z % nW:
            raise ValueError(f"window_mask must be [nW, {N}, {N}] with nW dividing {Z}")
    q8, k8, v8 = torch.empty((3, Z, H, N, D), dtype=torch.int8, device=dev).unbind(0)  # one allocation
    if out is None:
        out = torch.empty((Z, H, N, D), dtype=q.dtype, device=dev)
    ws = torch.empty(_lib.fused_workspace_bytes(nW if wm is not None else 1, H, N), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.fwd_fused_window(q, k, v, tab, idx, wm, nW, q8, k8, v8, out, scale * LOG2E, L_SHIFT, ACC_SHIFT,
                          arith_flags(), ws, stream)
    if check:
        st = _lib.fused_status(ws, stream)
        if st == 1:
            raise ZeroDivisionError("float division by zero (q or k is all zero)")
        if st == 3:
            raise IndexError("relative position index outside the bias table")
        if st != 0:
            raise ValueError("the fixed-point constants are not representable for this input")
    return out


def window_attention(query, key, value, rel_bias, window_mask=None, scale=None, return_mode='output'):
    """Swin window attention with the bias kept at window granularity.

    Equals ``qflash_forward(query, key, value, attn_mask=rel_bias + mask)``
    with the [B_, H, N, N] float mask that QWindowAttention builds
    (qflash/attention.py:68-74) -- bit for bit, because that mask's entry
    (b, h) is rel_bias[h] + window_mask[b % nW] and the bias quantisation is
    elementwise.  Here the sum and its quantisation are formed once per
    (window, head), [nW, H, N, N], and the kernel reads entry b % nW, so
    neither the expanded float mask nor the expanded int32 bias is built.

    query/key/value: [B_, H, N, D] with B_ a multiple of nW; rel_bias:
    [1, H, N, N]; window_mask: [nW, N, N] (0 / -100 shifted-window mask) or None.
    """
    if window_mask is None:
        return qflash_forward(query, key, value, rel_bias, scale, return_mode)
    nW, N = window_mask.shape[0], window_mask.shape[-1]
    if query.shape[0] % nW:
        raise ValueError(f"batch {query.shape[0]} is not a multiple of the {nW} windows")
    attn_mask = rel_bias + window_mask.view(nW, 1, N, N)
    if FUSED and return_mode == 'output' and _fused_takes(query, key, value, None) and attn_mask.is_cuda \
            and attn_mask.dtype in (torch.float32, torch.float16, torch.bfloat16):
        return forward_fused(query, key, value, attn_mask, scale, bias_z_period=nW, check=True)
    return forward_with_scales(query, key, value, attn_mask, scale, return_mode, bias_z_period=nW)


class qflash:
    """The reference's public op class (qflash/kernel.py:354-356)."""
    kernel = [launch_int8]
    forward = qflash_forward
