"""Multi-GPU execution of the attention forward: batch sharding.

(z, h) heads are independent, so each rank (one process per GPU) takes a
contiguous slice of the batch and runs the kernel on it with no data-path
communication.  The only subtlety is the per-tensor quantisation scale
(qflash/kernel.py:294-296): it is a max over the WHOLE tensor, so ranks
reduce their local |Q|, |K|, |V| maxima with one all_reduce(MAX) of three
scalars before quantising -- after that every shard's int8 values and
fixed-point constants are bit-identical to what a single process computes on
the full tensor.  ``gather=True`` collects the int8 outputs on every rank:
with a ``PeerOutput`` the attention epilogue itself stores every row into
every rank's copy of the gathered output over NVLink, and the kernel ends with
a barrier over the ranks (flags written into the peers' signal words, so the
kernel completes only once every copy is whole); otherwise NCCL all_gather
runs after the kernel.  Nothing else crosses GPUs.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import _lib
from .kernel import forward_with_scales, tensor_scales

MAX_RANKS = 8   # the epilogue stores into at most 7 peer copies
SIG_BYTES = 4 * _lib.SIG_WORDS  # signal words of the gather barrier and of the scale exchange


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of n units (sizes differ by at most one)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def global_scales(query, key, value, group=None, peer=None):
    """(q_scale, k_scale, o_scale) of the full tensors from this rank's shards.

    amax is exact under max-reduction; the values travel as fp32 (exact for
    fp16/bf16/fp32 inputs) and the division by 127 happens afterwards in the
    input dtype, as in the single-process path.  With ``peer`` (a PeerOutput)
    the maxima are exchanged through its signal words, else all_reduce."""
    dt = query.dtype
    local = torch.stack([t.abs().amax().to(torch.float32) for t in (query, key, value)])
    if peer is not None:
        local = peer.max_(local)
    elif dist.is_available() and dist.is_initialized():
        dist.all_reduce(local, op=dist.ReduceOp.MAX, group=group)
    i8max = torch.iinfo(torch.int8).max
    return tuple(local[i].to(dt) / i8max for i in range(3))


class _CudaArray:
    """A raw int8 device buffer exposed through ``__cuda_array_interface__``,
    which ``torch.as_tensor`` wraps without a copy."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "|i1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerOutput:
    """The gathered int8 output [Z, H, N, D] of a batch-sharded attention, one
    copy on every rank, mapped into every other rank's process (CUDA IPC), so
    that each rank's attention epilogue stores its shard's rows into all the
    copies at once (``qflash_i8_fwd_gather``).  Collective: every rank of
    ``group`` creates it with the same shape (on its current CUDA device) and
    calls ``close()``.  ``buffer`` is this rank's copy; a call of
    ``forward_sharded(..., gather=True, peer_out=...)`` overwrites it."""

    def __init__(self, shape, group=None):
        if not (dist.is_available() and dist.is_initialized()):
            raise RuntimeError("PeerOutput needs an initialised process group")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_RANKS:
            raise ValueError(f"{self.world} ranks: the fused gather takes at most {MAX_RANKS}")
        self.shape = tuple(int(x) for x in shape)
        if len(self.shape) != 4:
            raise ValueError("PeerOutput holds a [Z, H, N, D] tensor")
        self.device = torch.device("cuda", torch.cuda.current_device())
        # the int8 copy, then (256-byte aligned) the gather barrier's signal words
        self._sig_off = -(-math.prod(self.shape) // 256) * 256
        self._ptr, handle = _lib.ipc_alloc(self._sig_off + SIG_BYTES)
        self._epoch = 0
        self._max_epoch = 0
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self._peers = [_lib.ipc_open(h) for r, h in enumerate(handles) if r != self.rank]
        self.buffer = torch.as_tensor(_CudaArray(self._ptr, self.shape), device=self.device)
        if self.buffer.data_ptr() != self._ptr:
            raise RuntimeError("the gathered buffer was copied instead of wrapped")

    def peer_rows(self, z0: int) -> list[int]:
        """Addresses of batch entry z0 in every other rank's copy."""
        row = math.prod(self.shape[1:])
        return [p + z0 * row for p in self._peers]

    def next_barrier(self):
        """(sig, sig_peers, rank, epoch) for the next launch: every rank calls
        this once per launch, so the epochs agree."""
        self._epoch = self._epoch % 0x7fffffff + 1
        return (self._ptr + self._sig_off, [p + self._sig_off for p in self._peers], self.rank, self._epoch)

    def max_(self, values: torch.Tensor) -> torch.Tensor:
        """Max over the ranks of up to 4 float32 values on this rank's device
        (qflash_peer_max: written into every rank's signal words over NVLink,
        no library collective); NaN wins.  Collective: every rank calls it."""
        if values.dtype != torch.float32 or values.numel() > 4 or not values.is_cuda:
            raise ValueError("up to 4 float32 CUDA values")
        self._max_epoch = self._max_epoch % 0x7fffffff + 1
        inp = values.contiguous()
        out = torch.empty_like(inp)
        _lib.peer_max(inp, out, self._ptr + self._sig_off, [p + self._sig_off for p in self._peers], self.rank,
                      self._max_epoch, torch.cuda.current_stream(self.device).cuda_stream)
        return out

    def close(self):
        """Unmap the peers' copies and free this one (collective)."""
        if self._ptr is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)          # every rank's stores into every copy are done
        for p in self._peers:
            _lib.ipc_close(p)
        dist.barrier(group=self.group)          # no rank maps this copy any more
        self.buffer = None
        _lib.ipc_free(self._ptr)
        self._ptr, self._peers = None, []


def forward_sharded(query, key, value, attn_mask=None, scale=None, group=None, gather=False, launch=None,
                    peer_out: PeerOutput | None = None):
    """``qflash.forward`` on this rank's batch shard [Zl, H, N, D].

    attn_mask, if given, is this shard's mask (batch dimension sliced the same
    way, or broadcast with batch size 1).  Returns the dequantised local
    output, or with ``gather=True`` the full [Z, H, N, D] output assembled
    from every rank's int8 shard -- written by the attention epilogue into
    ``peer_out`` on every rank when given (shards in rank order), else
    collected with NCCL all_gather."""
    scales = global_scales(query, key, value, group, peer_out if gather else None)
    world = dist.get_world_size(group)
    if gather and peer_out is not None:
        sizes = torch.tensor([query.shape[0]], device=query.device)
        all_sizes = [torch.zeros_like(sizes) for _ in range(world)]
        dist.all_gather(all_sizes, sizes, group=group)
        all_sizes = [int(s.item()) for s in all_sizes]
        rank = dist.get_rank(group)
        z0 = sum(all_sizes[:rank])
        if peer_out.shape != (sum(all_sizes),) + tuple(query.shape[1:]):
            raise ValueError(f"peer_out holds {peer_out.shape}, the shards make "
                             f"{(sum(all_sizes),) + tuple(query.shape[1:])}")
        o_local = peer_out.buffer[z0:z0 + query.shape[0]]
        # the kernel completes only once every rank's rows are in every copy
        _, _, o_scale = forward_with_scales(query, key, value, attn_mask, scale, scales=scales, launch=launch,
                                            return_int8=True, o_out=o_local, o_peers=peer_out.peer_rows(z0),
                                            dequant=False, barrier=peer_out.next_barrier())
        return peer_out.buffer * o_scale
    out, o8, o_scale = forward_with_scales(query, key, value, attn_mask, scale, scales=scales,
                                           launch=launch, return_int8=True)
    if not gather:
        return out
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
