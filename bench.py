"""Benchmark of the integer-only attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload vit_b] [--impl ours|reference]

One step = one attention call (``qflash_i8_fwd``) over the whole workload, the
headline being the ViT-B/16 attention layer (B=256, H=12, N=197, d=64).
``value`` is int8 TOPS (4*Z*H*N^2*d ops per call) with the int8 inputs
resident in HBM; ``e2e`` is the same metric with the int8 Q/K/V copied from
pinned host memory and O copied back inside the timed region (steps pipelined
over copy-in, compute and copy-out streams).  With N > 1 GPUs
(launched by torchrun) every rank runs the full per-GPU workload on its own
GPU (weak scaling, no data-path collective) and the time is the max over ranks.

``--impl reference`` times the reference's integer algorithm on the host CPU
(the restatement in oracle/, all host cores, a bounded sample of heads of
the same workload), in the same metric.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def profile_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from a committed ncu summary, if one exists."""
    p = ROOT / "profiles" / f"{kernel}_{workload}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, interval_ms: int = 50):
        self.gpu = gpu_index
        self.interval = interval_ms
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 f"-lms={self.interval}"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r.split(", ") for r in self.out.strip().splitlines() if r.strip()]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if len(r) > 5 + i and "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        # the samples taken before the GPU ramped up are in the window too; use the upper half
        sm_sorted = sorted(sm)
        loaded = sm_sorted[len(sm_sorted) // 2:] if sm_sorted else []
        return {"sm_mhz": float(np.median(loaded)) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows)}


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    return rank, world, local


def cpu_sample_heads(q8, k8, v8, p, n_heads, seed=0):
    """Pick ``n_heads`` (z, h) heads of the workload for the CPU leg."""
    Z, H = q8.shape[:2]
    rng = np.random.default_rng(seed)
    idx = rng.choice(Z * H, size=min(n_heads, Z * H), replace=False)
    zs, hs = idx // H, idx % H
    return zs, hs


def _oracle_worker(args):
    q, k, v, prm, b = args
    from oracle import qflash_oracle as orc
    return orc.attention_int8(q, k, v, prm, b)


def run_cpu_oracle(q8n, k8n, v8n, prm, zs, hs, procs, bias=None):
    """Time the oracle on the sampled heads with ``procs`` worker processes
    (spawned; each head is an independent task)."""
    from oracle import qflash_oracle as orc
    tasks = [(q8n[z:z + 1, h:h + 1], k8n[z:z + 1, h:h + 1], v8n[z:z + 1, h:h + 1], prm,
              None if bias is None else bias[z:z + 1, h:h + 1]) for z, h in zip(zs, hs)]
    if procs <= 1:
        t0 = time.perf_counter()
        outs = [orc.attention_int8(*t) for t in tasks]
        return time.perf_counter() - t0, outs
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Pool(procs) as pool:
        pool.map(_oracle_worker, tasks[:procs])           # warm the workers
        t0 = time.perf_counter()
        outs = pool.map(_oracle_worker, tasks, chunksize=max(1, len(tasks) // (4 * procs)))
        dt = time.perf_counter() - t0
    return dt, outs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="vit_b")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline and parity sample (profiling runs)")
    a = ap.parse_args()
    if a.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    from qflash_b200.workloads import WORKLOADS
    w = WORKLOADS[a.workload]
    metric = f"int8 attn TOPS & us/call ({w.name} Z={w.Z} H={w.H} N={w.N} d={w.D}) and % of int8 TC/HBM roofline"
    rank, world, local = dist_setup(a.gpus)

    if a.impl == "reference":
        if rank != 0:
            return
        return bench_reference(a, w, metric)

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    from qflash_b200 import _lib
    from qflash_b200 import kernel as K
    from qflash_b200.workloads import make_inputs

    dev = torch.device("cuda", local)
    # inputs: the workload's float Q/K/V, quantised by the reference host path
    q, k, v, mask, win = make_inputs(w, seed=a.seed + rank, device=dev, parts=True)
    qs, ks, vs = (t.abs().amax() / 127 for t in (q, k, v))
    sm_scale, rs, eM, rM, lM, aM = K.fixed_point_params(float((qs * ks).item()), w.D, None)
    q8, k8, v8 = K.quantize(q, qs), K.quantize(k, ks), K.quantize(v, vs)
    bias, bstr, period = None, None, 0
    if win is not None:
        # Swin: the bias at window granularity, as QWindowAttention / window_attention use it
        rel, wmask = win
        if wmask is None:
            bias, bstr = K.quantize_bias(rel, sm_scale, w.Z, w.H, w.N)
        else:
            period = wmask.shape[0]
            bias, bstr = K.quantize_bias(rel + wmask.view(period, 1, w.N, w.N), sm_scale, period, w.H, w.N)
    del q, k, v, mask
    # rotating input sets so that no step finds its inputs in L2 (3 x 155 MB > 126 MB)
    n_sets = 3
    sets = [(q8, k8, v8, torch.empty_like(v8))]
    for i in range(1, n_sets):
        sets.append((q8.clone(), k8.clone(), v8.clone(), torch.empty_like(v8)))
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step(i):
        s = sets[i % n_sets]
        K.launch_int8(s[0], s[1], s[2], s[3], rs, eM, rM, lM, aM, bias, bstr, stream=sp, bias_z_period=period)

    for i in range(a.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = _lib.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(a.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - l0
    grid = _lib.last_grid()
    ms_total = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
        dist.barrier()
    torch.cuda.synchronize()
    ms_step = ms_total / a.steps
    assert _lib.device_error(sp) == 0

    # End to end through the C ABI: every step copies its int8 Q/K/V from pinned
    # host memory and reads its int8 O back, all inside the timed region.  The
    # steps are pipelined the way a server would run them: copy-in, attention
    # and copy-out on three streams over two device buffer sets, so step i's
    # host->device copy overlaps step i-1's kernel and device->host copy (PCIe
    # is full duplex).
    hq, hk, hv = (t.cpu().pin_memory() for t in (q8, k8, v8))
    ho = [torch.empty(v8.shape, dtype=torch.int8).pin_memory() for _ in range(2)]
    dbuf = [[torch.empty_like(q8) for _ in range(4)] for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_cmp = torch.cuda.Stream(dev)
    in_done = [torch.cuda.Event() for _ in range(2)]
    cmp_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    for ev in cmp_done + out_done:
        ev.record(stream)

    def e2e_step(i):
        b = i & 1
        dq, dk, dv, do = dbuf[b]
        s_in.wait_event(cmp_done[b])            # the kernel that read buffer b is done
        with torch.cuda.stream(s_in):
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            in_done[b].record(s_in)
        s_cmp.wait_event(in_done[b])
        s_cmp.wait_event(out_done[b])           # the copy that read output b is done
        K.launch_int8(dq, dk, dv, do, rs, eM, rM, lM, aM, bias, bstr, stream=s_cmp.cuda_stream,
                      bias_z_period=period)
        cmp_done[b].record(s_cmp)
        s_out.wait_event(cmp_done[b])
        with torch.cuda.stream(s_out):
            ho[b].copy_(do, non_blocking=True)
            out_done[b].record(s_out)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for st_ in (s_in, s_cmp, s_out):
        st_.wait_event(e0)
    for i in range(a.e2e_steps):
        e2e_step(i)
    for ev in out_done:
        stream.wait_event(ev)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / max(1, a.e2e_steps)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # The scaling runs' result collective, timed apart from the kernel: an NCCL
    # all_gather of every rank's int8 O shard (what forward_sharded(gather=True)
    # does); CUDA events on the current stream, max over ranks.
    gather = None
    if world > 1:
        o_loc = sets[0][3]
        parts = [torch.empty_like(o_loc) for _ in range(world)]
        for _ in range(2):
            dist.all_gather(parts, o_loc)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_g = 10
        g0.record(stream)
        for _ in range(n_g):
            dist.all_gather(parts, o_loc)
        g1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([g0.elapsed_time(g1) / n_g], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        g_ms = float(t.item())
        nb = o_loc.numel() * o_loc.element_size()
        gather = {"collective": "all_gather of the int8 O shards (NCCL)", "bytes_per_rank": int(nb),
                  "ms": round(g_ms, 4), "busbw_gbs": round(nb * (world - 1) / (g_ms * 1e-3) / 1e9, 1)}
        del parts

    # parity spot check and CPU baseline on a bounded sample of heads (rank 0, N=1 only)
    cpu = None
    sample_exact = None
    if rank == 0 and not a.no_cpu:
        from oracle import qflash_oracle as orc
        prm = orc.Params(sm_scale, rs, eM, rM, lM, aM)
        q8n, k8n, v8n = (t.cpu().numpy() for t in (q8, k8, v8))
        o_gpu = sets[0][3].cpu().numpy()
        bias_n = None
        if bias is not None:
            zb = period or (w.Z if bstr[0] else 1)
            bias_n = torch.as_strided(bias, (zb, w.H, w.N, w.N), bstr).cpu().numpy()
            if period:
                bias_n = bias_n[np.arange(w.Z) % period]
        zs, hs = cpu_sample_heads(q8n, k8n, v8n, prm, 2)
        t1, _ = run_cpu_oracle(q8n, k8n, v8n, prm, zs, hs, 1, bias_n)
        per_head = t1 / len(zs)
        nh = int(max(4, min(w.Z * w.H, a.cpu_seconds / max(per_head, 1e-6))))
        if world == 1:
            zs, hs = cpu_sample_heads(q8n, k8n, v8n, prm, nh, seed=1)
            dt, outs = run_cpu_oracle(q8n, k8n, v8n, prm, zs, hs, 1, bias_n)
            ops = 4 * len(zs) * w.N * w.N * w.D
            cpu = {"value": ops / dt / 1e12, "unit": "TOPS", "cores": 1, "kind": "port",
                   "sample": f"{len(zs)} of {w.Z * w.H} (z,h) heads of {w.name}, numpy oracle, 1 thread, {dt:.1f} s"}
            sample_exact = all(np.array_equal(o[0, 0], o_gpu[z, h]) for o, z, h in zip(outs, zs, hs))
        else:
            dt, outs = run_cpu_oracle(q8n, k8n, v8n, prm, zs, hs, 1, bias_n)
            sample_exact = all(np.array_equal(o[0, 0], o_gpu[z, h]) for o, z, h in zip(outs, zs, hs))

    ops_rank = w.ops
    value = ops_rank * world / (ms_step * 1e-3) / 1e12
    peaks, peak_src = load_peaks()
    bias_bytes = 0 if bias is None else int(bias.numel() * 4)   # read once per call (window granularity)
    bytes_launch = w.io_bytes + bias_bytes
    achieved = bytes_launch / (ms_step * 1e-3) / 1e9
    traffic = profile_traffic("qfa_fwd", w.name)
    clocks = clk.summary()
    if world > 1:
        import torch.distributed as dist  # noqa: F811
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": metric,
        "value": round(value, 3),
        "unit": "TOPS",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms_step, 6),
        "us_per_call": round(ms_step * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded N(0,1)-family inputs of the config's shape; see qflash_b200/workloads.py)",
        "config": {"workload": w.name, "Z": w.Z, "H": w.H, "N": w.N, "D": w.D, "bias_bytes": bias_bytes,
                   "l2": f"{n_sets} rotating input sets ({n_sets * w.io_bytes / 1e6:.0f} MB > 126 MB L2)",
                   "parallelism": f"dp{world} (per-GPU batch fixed)", "grid_ctas": grid},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                     "peak_source": peak_src,
                     "tc_frac": round(value / world / 4500.0, 4), "tc_peak_note": "4.5 POPS dense int8 (nominal)"},
        "e2e": {"value": round(ops_rank * world / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TOPS",
                "h2d_bytes_per_step": int(3 * w.Z * w.H * w.N * w.D), "d2h_bytes_per_step": int(w.Z * w.H * w.N * w.D),
                "path": "qflash_i8_fwd via ctypes, pinned host int8 buffers, copy-in / kernel / copy-out "
                        "pipelined on three streams"},
        "cpu_baseline": cpu,
        "gather": gather,
        "gpu_launches": int(launches),
        "clocks": clocks,
        "parity_sample_bit_exact": sample_exact,
    }
    print(json.dumps(line), flush=True)


def bench_reference(a, w, metric):
    """The reference's integer algorithm (oracle port) on all host cores."""
    import torch
    from oracle import qflash_oracle as orc
    from qflash_b200 import kernel as K
    from qflash_b200.workloads import make_inputs
    q, k, v, mask = make_inputs(w, seed=a.seed, device="cpu")
    qs, ks, vs = (t.abs().amax() / 127 for t in (q, k, v))
    sm_scale, rs, eM, rM, lM, aM = K.fixed_point_params(float((qs * ks).item()), w.D, None)
    q8n, k8n, v8n = (K.quantize(t, s).numpy() for t, s in ((q, qs), (k, ks), (v, vs)))
    bias_n = None
    if mask is not None:
        b, bstr = K.quantize_bias(mask, sm_scale, w.Z, w.H, w.N)
        bias_n = torch.as_strided(b, (w.Z, w.H, w.N, w.N), bstr).numpy()
    del q, k, v, mask
    prm = orc.Params(sm_scale, rs, eM, rM, lM, aM)
    procs = os.cpu_count() or 1
    # size one step to ~ a few seconds of all-core work
    zs, hs = cpu_sample_heads(q8n, k8n, v8n, prm, 2)
    t1, _ = run_cpu_oracle(q8n, k8n, v8n, prm, zs, hs, 1, bias_n)
    nh = int(max(procs, min(w.Z * w.H, 4.0 * procs / max(t1 / 2, 1e-6))))
    times = []
    for i in range(a.warmup + a.steps):
        zs, hs = cpu_sample_heads(q8n, k8n, v8n, prm, nh, seed=100 + i)
        dt, _ = run_cpu_oracle(q8n, k8n, v8n, prm, zs, hs, procs, bias_n)
        if i >= a.warmup:
            times.append(dt)
    dt = float(np.mean(times))
    ops = 4 * nh * w.N * w.N * w.D
    value = ops / dt / 1e12
    us_call = w.ops / (value * 1e12) * 1e6
    sample = f"{nh} of {w.Z * w.H} (z,h) heads per step, numpy oracle, {procs} processes"
    print(json.dumps({
        "metric": metric, "value": value, "unit": "TOPS", "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": dt * 1e3, "us_per_call": us_call, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic", "impl": "reference",
        "config": {"workload": w.name, "Z": w.Z, "H": w.H, "N": w.N, "D": w.D, "parallelism": "host CPU"},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": procs, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


if __name__ == "__main__":
    main()
