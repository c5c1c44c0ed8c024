"""Batch-sharded forward over 2 GPUs equals the single-GPU forward bit for bit,
with the result gathered by NCCL all_gather or by the attention epilogue's
stores into every rank's copy (PeerOutput)."""
import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path, fused):
    import torch.distributed as dist
    from qflash_b200.shard import PeerOutput, forward_sharded, shard_bounds
    from qflash_b200.workloads import WORKLOADS, make_inputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    w = WORKLOADS["vit_b"].scaled(7)
    q, k, v, _ = make_inputs(w, seed=3, device=dev)       # every rank builds the full tensors ...
    a, b = shard_bounds(w.Z, world, rank)                # ... and takes its batch slice
    peer = PeerOutput(q.shape) if fused else None
    outs = []
    for _ in range(2):   # a second call overwrites the gathered copies
        outs.append(forward_sharded(q[a:b].contiguous(), k[a:b].contiguous(), v[a:b].contiguous(), gather=True,
                                    peer_out=peer).cpu())
    torch.cuda.synchronize()
    from qflash_b200 import _lib
    assert _lib.device_error(torch.cuda.current_stream().cuda_stream) == 0
    torch.save(outs, os.path.join(path, f"r{rank}.pt"))
    if peer is not None:
        peer.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fused", [False, True], ids=["nccl_all_gather", "epilogue_peer_stores"])
def test_sharded_forward_two_gpus_bit_exact(fused):
    import torch.multiprocessing as mp
    from qflash_b200 import qflash
    from qflash_b200.workloads import WORKLOADS, make_inputs
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d, fused), nprocs=2, start_method="spawn", join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(2)]
    w = WORKLOADS["vit_b"].scaled(7)
    q, k, v, _ = make_inputs(w, seed=3, device="cuda:0")
    ref = qflash.forward(q, k, v).cpu()
    for per_rank in outs:
        for o in per_rank:
            assert torch.equal(o, ref)
