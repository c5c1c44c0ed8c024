"""Batch-sharded forward over 2 GPUs (NCCL) equals the single-GPU forward bit for bit."""
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


def _worker(rank, world, port, path):
    import torch.distributed as dist
    from qflash_b200.shard import forward_sharded, shard_bounds
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
    out = forward_sharded(q[a:b].contiguous(), k[a:b].contiguous(), v[a:b].contiguous(), gather=True)
    torch.cuda.synchronize()
    torch.save(out.cpu(), os.path.join(path, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_forward_two_gpus_bit_exact():
    import torch.multiprocessing as mp
    from qflash_b200 import qflash
    from qflash_b200.workloads import WORKLOADS, make_inputs
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(2, _free_port(), d), nprocs=2, start_method="spawn", join=True)
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(2)]
    w = WORKLOADS["vit_b"].scaled(7)
    q, k, v, _ = make_inputs(w, seed=3, device="cuda:0")
    ref = qflash.forward(q, k, v).cpu()
    for o in outs:
        assert torch.equal(o, ref)
