#!/usr/bin/env python
"""Benchmark of the sparse-mask attention hot path (pack_mask + fused masked
attention forward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1] [--impl ours|reference]

Multi-GPU runs are launched by torchrun (one process per GPU).  A step is one
``sparse_attention(q, k, v, mask)`` over one batch: pack the bool mask, then
the fused attention kernel (O and the FP32 LSE), inputs resident in HBM.
The L2 is flushed (512 MiB memset) before every step, outside the timed
events; each step is timed on its own with CUDA events and the p50 is taken,
then the max over ranks.  The two kernels are timed apart in a second pass
(an event between them; attn_ms_p50, pack_ms_p50 and the rooflines use it).

Default workload c1 (B16 H12 N512 D64 fp16, Bernoulli keep 0.25), the one the
reference quotes; with N GPUs every rank runs its own c1 batch (weak
scaling).  --config c5 splits the B*H heads of the large-batch workload
across ranks instead (strong scaling).

Prints ONE JSON line on rank 0.  --impl reference times the reference's CPU
implementation of the path (the oracle port, FP32 numpy) on this machine's
host cores on the same workload.
"""

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "sparse-mask-attention-auto-research_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "p50 latency ms & dense-equiv TFLOPS, B16H12N512D64 fp16 s=0.75, 1/2/4/8 B200"
UNIT = "TFLOPS (dense-equiv, 4*B*H*N^2*D / p50 step time)"
FLUSH_BYTES = 512 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", default="c1", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--pass", dest="which", default="forward", choices=["forward", "backward"],
                    help="backward: time sparse_attn_cuda.backward (one GPU) instead of the forward step")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm_gbs=p["hbm_gbs"], bf16_tflops=p["bf16_tflops"], source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, source="fallback")


def load_traffic(kernel, workload):
    """dram bytes per launch of `kernel` on `workload` from a committed ncu summary, else None."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        t = json.load(f)
    rec = t.get(f"{kernel}:{workload}")
    return None if rec is None else rec.get("dram_bytes_per_launch")


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.proc = None
        self.lines = []
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", uuid, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"], samples=0)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=smax, reasons=sorted(reasons),
                    samples=len(sm))


# ---------------------------------------------------------------- CPU (oracle port)


def cpu_step_fn(cfg_name, seed):
    """One pass of the oracle port (pack + FP32 attention) over the workload,
    all heads, threads over heads with single-threaded BLAS."""
    import numpy as np

    from oracle import oracle
    from python import workloads

    q, k, v, m = workloads.make_inputs(cfg_name, seed=seed, device="cpu")
    qf, kf, vf = (x.float().numpy() for x in (q, k, v))
    mf = m.numpy()
    D = q.shape[-1]
    threads = os.cpu_count() or 1

    def step():
        oracle.pack_mask_parallel(mf, threads=threads)
        oracle.attention_parallel(qf, kf, vf, mf, 1.0 / math.sqrt(D), threads=threads, with_lse=True)

    return step, threads, tuple(q.shape)


def time_cpu(cfg_name, seed, budget_s, min_reps=3, max_reps=30):
    from threadpoolctl import threadpool_limits

    step, threads, shape = cpu_step_fn(cfg_name, seed)
    times = []
    with threadpool_limits(limits=1):
        step()  # warm
        t_start = time.perf_counter()
        while len(times) < max_reps and (len(times) < min_reps or time.perf_counter() - t_start < budget_s):
            t0 = time.perf_counter()
            step()
            times.append(time.perf_counter() - t0)
    return statistics.median(times), threads, shape, len(times)


# ---------------------------------------------------------------- reference arm


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from python import workloads

    cfg = workloads.CONFIGS[args.config]
    from threadpoolctl import threadpool_limits

    step, threads, shape = cpu_step_fn(args.config, args.seed)
    B, H, N, D = shape
    flops = workloads.dense_flops(B, H, N, D)
    with threadpool_limits(limits=1):
        for _ in range(args.warmup):
            step()
        times = []
        t_all = time.perf_counter()
        for _ in range(args.steps):
            t0 = time.perf_counter()
            step()
            times.append(time.perf_counter() - t0)
        total = time.perf_counter() - t_all
    p50 = statistics.median(times)
    value = flops / p50 / 1e12
    sample = f"full {args.config} workload ({B*H} heads) per step: oracle pack + FP32 numpy attention with LSE"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": p50 * 1e3,
        "mean_ms": total / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/k/v, Bernoulli masks)",
        "config": {"workload": f"{args.config}: {workloads.describe(args.config)}", "global_batch": B, "seq_len": N,
                   "parallelism": "cpu threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm


def run_ours(args):
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 under torchrun")
    from python import SparseAttentionFunction, pack_mask, sparse_attention, sparse_attn_cuda, workloads
    from python.sparse_attention import _pack_for_attention as pack_for_attention

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = workloads.CONFIGS[args.config]
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    if args.config == "c5":
        scaling = "strong"
        BH = B * H
        lo, hi = BH * rank // world, BH * (rank + 1) // world
        q, k, v, m = workloads.make_inputs(args.config, seed=args.seed, device=dev, heads=(lo, hi))
        global_batch = B
    else:
        scaling = "weak"
        q, k, v, m = workloads.make_inputs(args.config, seed=args.seed + rank, device=dev)
        global_batch = B * world
    lb, lh = q.shape[0], q.shape[1]
    scale = 1.0 / math.sqrt(D)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step(evs=None):
        # Exactly sparse_attention(q, k, v, mask) for fp16/bf16 inputs
        # (python/sparse_attention.py).  With three events the two kernels are
        # also timed apart; an event between them costs the step a few µs (it
        # serialises the attention kernel's launch behind the packer), so the
        # step itself is timed with two.
        if evs:
            evs[0].record(stream)
        packed, occupancy = pack_for_attention(m, D)
        if evs and len(evs) == 3:
            evs[1].record(stream)
        out = SparseAttentionFunction.apply(q, k, v, packed, m, scale, N, occupancy)
        if evs:
            evs[-1].record(stream)
        return out

    # correctness guard: the bench path equals the public API
    ref_out = sparse_attention(q, k, v, m)
    assert torch.equal(step(), ref_out)
    for _ in range(args.warmup):
        flush.zero_()
        step()
    sparse_attn_cuda.device_status()

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    sampler = ClockSampler(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    t_wall = time.perf_counter()
    for i in range(args.steps):
        flush.zero_()
        step(evs[i])
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t_wall
    if world > 1:
        torch.distributed.barrier()
    clocks = sampler.stop()
    sparse_attn_cuda.device_status()

    step_ms = [e[0].elapsed_time(e[1]) for e in evs]
    # The two kernels timed apart, in a second pass of the same steps.
    split = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(min(args.steps, 500))]
    for i in range(len(split)):
        flush.zero_()
        step(split[i])
    torch.cuda.synchronize(dev)
    pack_ms = [e[0].elapsed_time(e[1]) for e in split]
    attn_ms = [e[1].elapsed_time(e[2]) for e in split]
    stats = torch.tensor([statistics.median(step_ms), statistics.fmean(step_ms), statistics.median(attn_ms),
                          statistics.fmean(attn_ms), statistics.median(pack_ms), statistics.fmean(pack_ms)],
                         dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
    p50_step, mean_step, p50_attn, mean_attn, p50_pack, mean_pack = stats.tolist()

    # Optional NVLink gather of the output shards (timed separately; not part of a step).
    gather_ms = None
    if world > 1:
        out = step()
        gathered = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=dev)
        for _ in range(3):
            torch.distributed.all_gather_into_tensor(gathered, out)
        torch.cuda.synchronize(dev)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(10):
            torch.distributed.all_gather_into_tensor(gathered, out)
        g1.record(stream)
        torch.cuda.synchronize(dev)
        gt = torch.tensor([g0.elapsed_time(g1) / 10], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(gt, op=torch.distributed.ReduceOp.MAX)
        gather_ms = gt.item()
        del gathered

    # End to end through the public API from pinned host memory.
    e2e = None
    if args.e2e_steps > 0:
        hq, hk, hv, hm = (x.cpu().pin_memory() for x in (q, k, v, m))
        dq, dk, dv, dm = (torch.empty_like(x) for x in (q, k, v, m))
        hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        e_times = []
        for i in range(args.e2e_steps + 3):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            dm.copy_(hm, non_blocking=True)
            o = sparse_attention(dq, dk, dv, dm)
            hout.copy_(o, non_blocking=True)
            b.record(stream)
            b.synchronize()
            if i >= 3:
                e_times.append(a.elapsed_time(b))
        et = torch.tensor([statistics.median(e_times)], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(et, op=torch.distributed.ReduceOp.MAX)
        flops_all = workloads.dense_flops(lb, lh, N, D) * world
        e2e = {"value": flops_all / (et.item() * 1e-3) / 1e12, "unit": UNIT, "p50_ms": et.item(),
               "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in (hq, hk, hv, hm)),
               "d2h_bytes_per_step": hout.numel() * hout.element_size()}
        assert torch.equal(hout, ref_out.cpu())

    # CPU baseline (oracle port) on rank 0 at N=1 only.
    cpu_baseline = None
    if world == 1 and not args.no_cpu_baseline and args.config != "c5":
        t, threads, shape, reps = time_cpu(args.config, args.seed, args.cpu_seconds)
        b_, h_, n_, d_ = shape
        cpu_baseline = {"value": workloads.dense_flops(b_, h_, n_, d_) / t / 1e12, "unit": UNIT, "cores": threads,
                        "kind": "port", "ms": t * 1e3,
                        "sample": f"full {args.config} workload ({b_*h_} heads), oracle pack + FP32 numpy attention "
                                  f"with LSE, p50 of {reps} runs"}

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0

    peaks = load_peaks()
    # Both head dims run the persistent two-chain kernel.
    attn_kernel = "attn_fwd_chain_kernel"
    bm, bn = workloads.kernel_tile(D)
    live = workloads.live_tile_fraction(m, bm, bn)
    a_bytes = workloads.attn_bytes(lb, lh, N, D)
    achieved_gbs = a_bytes / (mean_attn * 1e-3) / 1e9
    tflops_live = workloads.live_flops(lb, lh, N, D, live, bm, bn) / (mean_attn * 1e-3) / 1e12
    p_bytes = workloads.pack_bytes(lb, lh, N)
    flops_step = workloads.dense_flops(lb, lh, N, D)
    value = flops_step * world / (p50_step * 1e-3) / 1e12
    workload = f"{args.config}: {workloads.describe(args.config)}" + (" per rank" if scaling == "weak" else " split over ranks")
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": p50_step,
        "mean_ms_per_step": mean_step,
        "attn_ms_p50": p50_attn,
        "pack_ms_p50": p50_pack,
        "higher_is_better": True,
        "scaling": scaling,
        "vs_baseline": None,
        "dtype": {torch.float16: "fp16", torch.bfloat16: "bf16"}[cfg["dtype"]],
        "data": "synthetic (seeded N(0,1) q/k/v, seeded masks per the workload recipe)",
        "config": {"workload": workload, "global_batch": global_batch, "seq_len": N, "heads": H, "head_dim": D,
                   "parallelism": f"bh-shard{world}" if world > 1 else "single",
                   "l2": "flushed (512 MiB memset) before every timed step"},
        "roofline": {"bound": "hbm", "achieved": achieved_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved_gbs / peaks["hbm_gbs"], "traffic": load_traffic(attn_kernel, args.config),
                     "kernel": attn_kernel, "algorithmic_bytes_per_launch": a_bytes,
                     "avg_launch_ms": mean_attn, "peak_source": peaks["source"]},
        "roofline_tensor": {"achieved": tflops_live, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                            "frac": tflops_live / peaks["bf16_tflops"], "live_tile_fraction": live,
                            "tile": [bm, bn]},
        "pack_roofline": {"achieved": p_bytes / (mean_pack * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": p_bytes / (mean_pack * 1e-3) / 1e9 / peaks["hbm_gbs"]},
        "clocks": clocks,
        "gpu_launches": 2 * args.steps,
        "split_pass_steps": len(split),
        "timed_wall_s": wall,
    }
    if gather_ms is not None:
        line["gather_ms"] = gather_ms
    if e2e is not None:
        line["e2e"] = e2e
    if cpu_baseline is not None:
        line["cpu_baseline"] = cpu_baseline
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def run_backward(args):
    """One GPU: the backward (dq, dk, dv from dout and the forward's out and
    lse) on the workload, inputs resident in HBM, L2 flushed before every
    step.  Prints one JSON line in the forward's format."""
    rank, world, local = dist_env()
    if world != 1 or args.gpus != 1:
        raise SystemExit("--pass backward runs on one GPU")
    from python import pack_mask, sparse_attn_cuda, workloads

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = workloads.CONFIGS[args.config]
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    q, k, v, m = workloads.make_inputs(args.config, seed=args.seed, device=dev)
    g = torch.Generator(device=dev).manual_seed(args.seed + 7)
    dout = torch.randn(q.shape, generator=g, device=dev).to(q.dtype)
    scale = 1.0 / math.sqrt(D)
    packed = pack_mask(m)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=dev, dtype=torch.float32)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, scale, True)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        sparse_attn_cuda.backward(dout, q, k, v, out, lse, packed, dq, dk, dv, scale)

    for _ in range(args.warmup):
        flush.zero_()
        step()
    sparse_attn_cuda.device_status()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    sampler = ClockSampler(dev)
    torch.cuda.synchronize(dev)
    for i in range(args.steps):
        flush.zero_()
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    sparse_attn_cuda.device_status()
    ms = sorted(e[0].elapsed_time(e[1]) for e in evs)
    p50 = ms[len(ms) // 2]
    peaks = load_peaks()
    flops = workloads.backward_flops(B, H, N, D)
    nbytes = workloads.backward_bytes(B, H, N, D)
    live = workloads.live_tile_fraction(m, 128, 128)
    mma_flops = flops * live  # the kernel's five products run on live 128x128 tile pairs only
    line = {
        "metric": "backward dense-equiv TFLOPS (10*B*H*N^2*D / p50 step)",
        "value": flops / (p50 * 1e-3) / 1e12,
        "unit": "TFLOPS",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": p50,
        "higher_is_better": True,
        "dtype": {torch.float16: "fp16", torch.bfloat16: "bf16"}[cfg["dtype"]],
        "data": "synthetic (seeded N(0,1) q/k/v/dout, seeded masks per the workload recipe)",
        "config": {"workload": f"{args.config}: {workloads.describe(args.config)}", "pass": "backward",
                   "l2": "flushed (512 MiB memset) before every timed step"},
        "roofline": {"bound": "hbm", "achieved": nbytes / (p50 * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": nbytes / (p50 * 1e-3) / 1e9 / peaks["hbm_gbs"],
                     "algorithmic_bytes_per_step": nbytes, "peak_source": peaks["source"]},
        "roofline_tensor": {"achieved": mma_flops / (p50 * 1e-3) / 1e12, "peak": peaks["bf16_tflops"],
                            "unit": "TFLOP/s", "frac": mma_flops / (p50 * 1e-3) / 1e12 / peaks["bf16_tflops"],
                            "live_tile_fraction": live},
        "clocks": clocks,
        "gpu_launches": 3 * args.steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.which == "backward":
        return run_backward(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
