"""Multi-rank host path (qflash_b200.shard) on CPU with gloo, world size 2.

The kernel launch is replaced by a stub that copies V to O, so these tests
cover the sharding, the global scales, quantisation and the gather -- the
logic around the kernel, which the GPU tests cover on its own."""
import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qflash_b200 import kernel as K
from qflash_b200.shard import forward_sharded, global_scales, shard_bounds


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stub(captured):
    def launch(q8, k8, v8, o8, rs, eM, rM, lM, aM, bias=None, bs=None):
        captured.update(q8=q8.clone(), k8=k8.clone(), v8=v8.clone(), params=(rs, eM, rM, lM, aM),
                        bias=None if bias is None else torch.as_strided(bias, (q8.shape[0], q8.shape[1], q8.shape[2],
                                                                              q8.shape[2]), bs).clone())
        o8.copy_(v8)
    return launch


def _worker(rank, world, port, path, dtype, Z, with_mask):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(Z, 3, 40, 32, generator=g).to(dtype) for _ in range(3))
    mask = torch.randn(Z, 3, 40, 40, generator=g) if with_mask else None
    a, b = shard_bounds(Z, world, rank)
    cap = {}
    out = forward_sharded(q[a:b], k[a:b], v[a:b], None if mask is None else mask[a:b], gather=True,
                          launch=_stub(cap))
    torch.save({"out": out, "cap": cap, "bounds": (a, b)}, os.path.join(path, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("dtype,Z,with_mask", [(torch.float32, 5, False), (torch.float16, 4, False),
                                               (torch.float32, 3, True)])
def test_sharded_host_path_matches_single_process(dtype, Z, with_mask):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d, dtype, Z, with_mask), nprocs=world,
                           start_method="spawn", join=True)
        res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(Z, 3, 40, 32, generator=g).to(dtype) for _ in range(3))
    mask = torch.randn(Z, 3, 40, 40, generator=g) if with_mask else None
    cap = {}
    full = K.forward_with_scales(q, k, v, mask, launch=_stub(cap))
    for r in res:
        a, b = r["bounds"]
        assert r["cap"]["params"] == cap["params"]
        for name in ("q8", "k8", "v8"):
            assert torch.equal(r["cap"][name], cap[name][a:b])
        if with_mask:
            assert torch.equal(r["cap"]["bias"], cap["bias"][a:b])
        assert torch.equal(r["out"], full)  # gathered output, in batch order


def test_shard_bounds_partition():
    for n in (0, 1, 5, 256, 1023):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def test_global_scales_single_process_equal_tensor_scales():
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(2, 2, 8, 32, generator=g).half() for _ in range(3))
    for a, b in zip(global_scales(q, k, v), K.tensor_scales(q, k, v)):
        assert a.dtype == b.dtype and torch.equal(a, b)


def _dead_peer_worker(rank, world, port, path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)                      # leaves without joining the scale reduction
    q = torch.randn(1, 1, 8, 32)
    try:
        forward_sharded(q, q, q, launch=_stub({}))
        outcome = "completed"
    except Exception as e:               # the collective must fail, not hang
        outcome = f"raised {type(e).__name__}"
    with open(os.path.join(path, "r0.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_dead_peer_raises_instead_of_hanging():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_dead_peer_worker, args=(2, _free_port(), d), nprocs=2, start_method="spawn",
                                 join=False)
        for p in ctx.processes:
            p.join(timeout=60)
        alive = [p for p in ctx.processes if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank hung"
        with open(os.path.join(d, "r0.txt")) as f:
            assert f.read().startswith("raised")


def test_peer_output_needs_a_process_group():
    from qflash_b200.shard import PeerOutput
    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    with pytest.raises(RuntimeError, match="process group"):
        PeerOutput((2, 3, 40, 32))


class _FakePeerOutput:
    """Stands in for shard.PeerOutput on CPU: the gathered copy is a plain
    tensor, the scale exchange a gloo all_reduce, and the launch stub below
    plays the epilogue's peer stores with an all_gather."""

    def __init__(self, shape):
        self.shape = tuple(shape)
        self.buffer = torch.full(self.shape, 99, dtype=torch.int8)
        self.epochs = []

    def peer_rows(self, z0):
        return [z0]

    def next_barrier(self):
        self.epochs.append(len(self.epochs) + 1)
        return (0, [], dist.get_rank(), self.epochs[-1])

    def max_(self, values):
        out = values.clone()
        dist.all_reduce(out, op=dist.ReduceOp.MAX)
        return out


def _peer_stub(peer, sizes):
    def launch(q8, k8, v8, o8, rs, eM, rM, lM, aM, bias=None, bs=None):
        z0 = sum(sizes[:dist.get_rank()])              # this rank's rows sit at its batch offset
        assert o8.data_ptr() == peer.buffer[z0].data_ptr() and o8.shape[0] == sizes[dist.get_rank()]
        o8.copy_(v8)                                   # the local rows, written into the gathered copy
        zmax = max(sizes)                              # every other rank's rows, as its epilogue stores them
        mine = torch.zeros((zmax,) + tuple(o8.shape[1:]), dtype=torch.int8)
        mine[:o8.shape[0]] = o8
        parts = [torch.zeros_like(mine) for _ in sizes]
        dist.all_gather(parts, mine)
        peer.buffer.copy_(torch.cat([p[:n] for p, n in zip(parts, sizes)]))
    return launch


def _peer_worker(rank, world, port, path, Z):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(Z, 3, 40, 32, generator=g) for _ in range(3))
    a, b = shard_bounds(Z, world, rank)
    sizes = [e - s for s, e in (shard_bounds(Z, world, r) for r in range(world))]
    peer = _FakePeerOutput(q.shape)
    outs = [forward_sharded(q[a:b], k[a:b], v[a:b], gather=True, launch=_peer_stub(peer, sizes), peer_out=peer)
            for _ in range(2)]
    bad = None
    try:
        forward_sharded(q[a:b], k[a:b], v[a:b], gather=True, launch=_peer_stub(peer, sizes),
                        peer_out=_FakePeerOutput((Z + 1,) + tuple(q.shape[1:])))
    except ValueError as e:
        bad = str(e)
    torch.save({"outs": outs, "epochs": peer.epochs, "bad": bad}, os.path.join(path, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("Z", [4, 5])
def test_sharded_forward_with_peer_output_host_logic(Z):
    """forward_sharded(gather=True, peer_out=...): global scales through the
    peer exchange, this rank's rows at its batch offset of the gathered copy,
    one barrier epoch per call, the dequantised whole output on every rank,
    and a copy of the wrong shape rejected."""
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_peer_worker, args=(world, _free_port(), d, Z), nprocs=world, start_method="spawn",
                           join=True)
        res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(Z, 3, 40, 32, generator=g) for _ in range(3))
    full = K.forward_with_scales(q, k, v, launch=_stub({}))
    for r in res:
        assert r["epochs"] == [1, 2]
        for o in r["outs"]:
            assert torch.equal(o, full)
        assert r["bad"] is not None and "peer_out holds" in r["bad"]
