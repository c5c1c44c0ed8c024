"""Multi-GPU execution of the attention forward: batch sharding.

(z, h) heads are independent, so each rank (one process per GPU) takes a
contiguous slice of the batch and runs the kernel on it with no data-path
communication.  The only subtlety is the per-tensor quantisation scale
(qflash/kernel.py:294-296): it is a max over the WHOLE tensor, so ranks
reduce their local |Q|, |K|, |V| maxima with one all_reduce(MAX) of three
scalars before quantising -- after that every shard's int8 values and
fixed-point constants are bit-identical to what a single process computes on
the full tensor.  ``gather=True`` collects the int8 outputs on every rank
with all_gather (the result a scaling run checks); nothing else crosses GPUs.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .kernel import forward_with_scales, tensor_scales


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of n units (sizes differ by at most one)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def global_scales(query, key, value, group=None):
    """(q_scale, k_scale, o_scale) of the full tensors from this rank's shards.

    amax is exact under max-reduction; the values travel as fp32 (exact for
    fp16/bf16/fp32 inputs) and the division by 127 happens afterwards in the
    input dtype, as in the single-process path."""
    dt = query.dtype
    local = torch.stack([t.abs().amax().to(torch.float32) for t in (query, key, value)])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(local, op=dist.ReduceOp.MAX, group=group)
    i8max = torch.iinfo(torch.int8).max
    return tuple(local[i].to(dt) / i8max for i in range(3))


def forward_sharded(query, key, value, attn_mask=None, scale=None, group=None, gather=False, launch=None):
    """``qflash.forward`` on this rank's batch shard [Zl, H, N, D].

    attn_mask, if given, is this shard's mask (batch dimension sliced the same
    way, or broadcast with batch size 1).  Returns the dequantised local
    output, or with ``gather=True`` the full [Z, H, N, D] output assembled
    from every rank's int8 shard."""
    scales = global_scales(query, key, value, group)
    out, o8, o_scale = forward_with_scales(query, key, value, attn_mask, scale, scales=scales,
                                           launch=launch, return_int8=True)
    if not gather:
        return out
    world = dist.get_world_size(group)
    sizes = torch.tensor([o8.shape[0]], device=o8.device)
    all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
    dist.all_gather(all_sizes, sizes, group=group)
    zmax = int(max(int(s.item()) for s in all_sizes))
    padded = o8.new_zeros((zmax,) + tuple(o8.shape[1:]))
    padded[: o8.shape[0]] = o8
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded.contiguous(), group=group)
    full = torch.cat([p[: int(s.item())] for p, s in zip(parts, all_sizes)], dim=0)
    return full * o_scale
