#!/usr/bin/env python
"""Benchmark of the sparse-mask attention hot path (pack_mask + fused masked
attention forward) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1]
                    [--impl ours|reference|reference_cuda] [--pass forward|backward]

Multi-GPU runs are launched by torchrun (one process per GPU).  A step is one
``sparse_attention(q, k, v, mask)`` over one batch: pack the bool mask, then
the fused attention kernel (O and the FP32 LSE), inputs resident in HBM.
Before every timed step the L2 is flushed: a 512 MiB memset, then a 256 MiB
read, so that no input is in L2 and the lines left there are clean (the
state ncu's cache control gives a kernel).  Each step is timed on its own
with CUDA events on the launching stream and the p50 is taken, then the max
over ranks.  The two kernels are timed apart in a second pass (an event
between them; attn_ms_p50, pack_ms_p50 and the rooflines use it).

Headline workload c1 (B16 H12 N512 D64 fp16, Bernoulli keep 0.25): with N
GPUs every rank runs its own c1 batch (weak scaling, `value`).  Every line
also carries `strong_c5`: the large-batch workload c5 (B256 H16 N512 D64)
split by batch*head over the N ranks, max-over-ranks step time, and its
efficiency against one GPU running all of c5 in the same run.  The one-GPU
line adds `configs` (c1..c5 step, attention and roofline figures),
`backward` (the backward kernel on c1) and `sweep` (the reference's own
performance sweep, run.py:483-540: N from 64 to 16384 and B from 1 to 64).

Prints ONE JSON line on rank 0.  --impl reference times the reference's own
CPU implementation of the path (its torch masked-softmax attention,
restated in oracle/torch_ref.py) on this machine's host cores with every
thread, on the same workload and config.  --impl reference_cuda times the
reference's own CUDA kernels (pack + scalar forward, built from its sources
into oracle/_ref/) the way its run.py does, on c1..c5.
"""

import argparse
import ctypes
import datetime
import json
import math
import os
import statistics
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
CLEAN_BYTES = 256 << 20
L2_NOTE = ("GPU arms: L2 flushed before every timed step (512 MiB memset, then a 256 MiB read so no input "
           "is in L2 and the lines left are clean)")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="c1", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_cuda"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--block-steps", type=int, default=50,
                    help="timed steps of each sub-block (strong_c5, configs, backward)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-blocks", action="store_true", help="headline only (no strong_c5/configs/backward)")
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


def workload_config(name, world, weak):
    """The `config` object of every arm's line for workload `name` at `world` ranks."""
    from python import workloads

    c = workloads.CONFIGS[name]
    return {"workload": f"{name}: {workloads.describe(name)}" + (" per rank" if weak else " split over ranks"),
            "global_batch": c["B"] * world if weak else c["B"], "seq_len": c["N"], "heads": c["H"],
            "head_dim": c["D"], "parallelism": f"bh-shard{world}" if world > 1 else "single", "l2": L2_NOTE}


# ---------------------------------------------------------------- clocks


class ClockSampler:
    """Polls the GPU's SM clock and clock-event (throttle) reasons through
    NVML every ~0.25 ms from a background thread (query only).  `mark()`
    brackets the timed region; `report()` summarises the samples inside it
    and, separately, all samples of the run."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        self.samples = []
        self.windows = {}
        self.stop_ev = threading.Event()
        self.err = None
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            getter = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.reasons_fn = getter
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception as e:  # no NVML: report that instead of clocks
            self.err = f"nvml unavailable: {e}"
            self.h = None

    def _run(self):
        nv = self.nv
        while not self.stop_ev.is_set():
            try:
                t = time.perf_counter()
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                reasons = self.reasons_fn(self.h)
                self.samples.append((t, mhz, reasons))
            except Exception as e:
                self.err = str(e)
                return
            time.sleep(0.00025)

    def mark(self, name, t0, t1):
        self.windows[name] = (t0, t1)

    def stop(self):
        """Ends the polling (the samples are kept for report()): a thread
        that takes the GIL every 0.25 ms slows host-heavy work timed later,
        such as the streamed end-to-end copies."""
        self.stop_ev.set()
        if self.h is not None:
            self.thread.join(timeout=2)

    def _summary(self, samples):
        if not samples:
            return dict(sm_mhz=None, samples=0, reasons=[])
        reasons = set()
        for _, _, r in samples:
            for bit, name in self.REASONS.items():
                if r & bit:
                    reasons.add(name)
        return dict(sm_mhz=statistics.median(s[1] for s in samples), samples=len(samples), reasons=sorted(reasons))

    def report(self, window):
        self.stop()
        if self.h is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=[self.err], samples=0)
        t0, t1 = self.windows.get(window, (0.0, 0.0))
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        out = self._summary(inside)
        out["sm_max_mhz"] = self.max_mhz
        out["window"] = "timed steps only (NVML, query-only polling every ~0.25 ms)"
        whole = self._summary(self.samples)
        # Every sample taken: warm-up and timed steps (polling stops after them).
        out["whole_run"] = dict(sm_mhz=whole["sm_mhz"], samples=whole["samples"], reasons=whole["reasons"])
        if self.err:
            out["error"] = self.err
        return out


# ---------------------------------------------------------------- timing helpers


class Flusher:
    """L2 flush before each timed step: a write larger than L2, then a read
    that leaves clean lines."""

    def __init__(self, dev):
        self.buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.clean = torch.ones(CLEAN_BYTES // 8, dtype=torch.int64, device=dev)
        self.sink = torch.empty((), dtype=torch.int64, device=dev)

    def __call__(self, dirty=False):
        self.buf.zero_()
        if not dirty:
            torch.sum(self.clean, dim=0, out=self.sink)


def time_steps(fn, n, flush, stream, marks=1, dirty=False):
    """Runs `fn(events)` n times after a flush each; fn records len(events)
    events.  Returns the per-step list of event gaps [(e1-e0, e2-e1, ...)]."""
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(marks + 1)] for _ in range(n)]
    for i in range(n):
        flush(dirty=dirty)
        fn(evs[i])
    torch.cuda.synchronize()
    return [[e[j].elapsed_time(e[j + 1]) for j in range(marks)] for e in evs]


def p50(xs):
    return statistics.median(xs)


def back_to_back_ms(fn, stream, warmup=10, repeat=50):
    """The reference's own timing (run.py:206-217): `repeat` back-to-back
    calls between two events after `warmup`, no flush, the mean per call."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(repeat):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / repeat


def max_over_ranks(vals, dev, world):
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return t.tolist()


# ---------------------------------------------------------------- the forward step


class ForwardStep:
    """sparse_attention(q, k, v, mask) for fp16/bf16 inputs
    (python/sparse_attention.py), with hooks for events between the two
    kernels."""

    def __init__(self, q, k, v, m):
        from python import SparseAttentionFunction
        from python.sparse_attention import _pack_for_attention

        self.fn = SparseAttentionFunction
        self.pack = _pack_for_attention
        self.q, self.k, self.v, self.m = q, k, v, m
        self.D = q.shape[-1]
        self.N = q.shape[2]
        self.scale = 1.0 / math.sqrt(self.D)
        self.stream = torch.cuda.current_stream(q.device)

    def __call__(self, evs=None):
        # With three events the two kernels are also timed apart; an event
        # between them costs the step a few µs (it serialises the attention
        # kernel's launch behind the packer), so the step itself is timed
        # with two.
        if evs:
            evs[0].record(self.stream)
        packed, occupancy = self.pack(self.m, self.D)
        if evs and len(evs) == 3:
            evs[1].record(self.stream)
        out = self.fn.apply(self.q, self.k, self.v, packed, self.m, self.scale, self.N, occupancy)
        if evs:
            evs[-1].record(self.stream)
        return out


def attn_roofline(name, lb, lh, N, D, m, attn_ms_mean, peaks):
    """The attention kernel's roofline figures: algorithmic bytes at HBM
    bandwidth and live-tile MMA FLOPs at tensor peak; the slower of the two
    bounds the kernel."""
    from python import workloads

    bm, bn = workloads.kernel_tile(D)
    live = workloads.live_tile_fraction(m, bm, bn)
    live_canon = workloads.live_tile_fraction(m, 128, 64)
    a_bytes = workloads.attn_bytes(lb, lh, N, D)
    flops = workloads.live_flops(lb, lh, N, D, live, bm, bn)
    t = attn_ms_mean * 1e-3
    hbm_us = a_bytes / (peaks["hbm_gbs"] * 1e9) * 1e6
    mma_us = flops / (peaks["bf16_tflops"] * 1e12) * 1e6
    bound = "hbm" if hbm_us >= mma_us else "tensor"
    return {"bound": bound, "frac": max(hbm_us, mma_us) / (t * 1e6), "hbm_bound_us": hbm_us, "mma_bound_us": mma_us,
            "hbm_frac": a_bytes / t / 1e9 / peaks["hbm_gbs"], "tensor_frac": flops / t / 1e12 / peaks["bf16_tflops"],
            "achieved_gbs": a_bytes / t / 1e9, "achieved_tflops": flops / t / 1e12,
            "algorithmic_bytes_per_launch": a_bytes, "live_tile_fraction": live, "tile": [bm, bn],
            "live_tile_fraction_128x64": live_canon}


def measure_forward(name, dev, flush, steps, seed, heads=None, with_split=True):
    """p50 / mean step and split times of the forward on workload `name` (or
    a workload config dict), optionally a slice of its flattened batch*head
    range."""
    from python import workloads

    q, k, v, m = workloads.make_inputs(name, seed=seed, device=dev, heads=heads)
    step = ForwardStep(q, k, v, m)
    for _ in range(3):
        flush()
        step()
    st = [s[0] for s in time_steps(step, steps, flush, step.stream, marks=1)]
    res = {"step_ms_p50": p50(st), "step_ms_mean": statistics.fmean(st), "q": q, "m": m}
    if with_split:
        sp = time_steps(step, steps, flush, step.stream, marks=2)
        res.update(pack_ms_p50=p50([s[0] for s in sp]), attn_ms_p50=p50([s[1] for s in sp]),
                   pack_ms_mean=statistics.fmean([s[0] for s in sp]),
                   attn_ms_mean=statistics.fmean([s[1] for s in sp]))
    return res


# ---------------------------------------------------------------- CPU reference path


def cpu_reference_step(cfg_name, seed):
    """One pass of the reference's own CPU path (oracle/torch_ref.py) over the
    workload, all heads, every host thread."""
    from oracle import torch_ref
    from python import workloads

    q, k, v, m = workloads.make_inputs(cfg_name, seed=seed, device="cpu")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def step():
        return torch_ref.sparse_attention_cpu(q, k, v, m)

    return step, threads, tuple(q.shape)


def time_cpu(cfg_name, seed, budget_s, min_reps=3, max_reps=30):
    step, threads, shape = cpu_reference_step(cfg_name, seed)
    step()  # warm
    times = []
    t_start = time.perf_counter()
    while len(times) < max_reps and (len(times) < min_reps or time.perf_counter() - t_start < budget_s):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    return p50(times), threads, shape, len(times)


def cpu_sample_text(name, B, H, reps=None):
    s = (f"full {name} workload ({B * H} heads) per step: the reference's CPU path "
         "sparse_attention() -> sparse_attention_ref in FP32 torch (python/sparse_attention.py:26-44, :150-151), "
         "restated in oracle/torch_ref.py")
    return s + (f", p50 of {reps} runs" if reps else "")


# ---------------------------------------------------------------- reference arm (CPU)


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from python import workloads

    step, threads, shape = cpu_reference_step(args.config, args.seed)
    B, H, N, D = shape
    flops = workloads.dense_flops(B, H, N, D)
    for _ in range(args.warmup):
        step()
    times = []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    total = time.perf_counter() - t_all
    t50 = p50(times)
    value = flops / t50 / 1e12
    sample = cpu_sample_text(args.config, B, H)
    weak = args.config != "c5"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t50 * 1e3,
        "mean_ms_per_step": total / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak" if weak else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/k/v, seeded masks per the workload recipe)",
        "config": workload_config(args.config, args.gpus, weak),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
                         "torch_threads": torch.get_num_threads()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "one rank (rank 0) runs the CPU path; the workload per step is one rank's batch",
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- reference arm (its CUDA kernels)


def run_reference_cuda(args):
    """The reference's own pack_mask + scalar forward kernels, built from its
    sources into oracle/_ref/libref_sma.so, timed the way its run.py times
    sparse_attention_cuda_fwd (run.py:157-168, is_training=False): a zeroed
    packed buffer (binding.cpp:56-57), the pack kernel, then the forward."""
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    lib_path = os.path.join(REPO, "oracle", "_ref", "libref_sma.so")
    if not os.path.exists(lib_path):
        print(json.dumps({"impl": "reference_cuda", "unavailable": "oracle/_ref/libref_sma.so not built"}))
        return 0
    from python import workloads

    lib = ctypes.CDLL(lib_path)
    vp = ctypes.c_void_p
    lib.ref_pack_mask.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp]
    lib.ref_attn_fwd.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp] + [ctypes.c_int] * 4 + [ctypes.c_float,
                                                                                               ctypes.c_int, vp]
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    flush = Flusher(dev)
    stream = torch.cuda.current_stream(dev)
    peaks = load_peaks()
    results = {}
    for name in ("c1", "c2", "c3", "c4", "c5"):
        q, k, v, m = workloads.make_inputs(name, seed=args.seed, device=dev)
        B, H, N, D = q.shape
        packed = torch.zeros(B, H, N, (N + 31) // 32, dtype=torch.int32, device=dev)
        out = torch.empty_like(q)
        lse = torch.empty(B, H, N, dtype=torch.float32, device=dev)
        bf = 1 if q.dtype == torch.bfloat16 else 0

        def step(evs):
            evs[0].record(stream)
            packed.zero_()
            assert lib.ref_pack_mask(m.data_ptr(), packed.data_ptr(), B, H, N, stream.cuda_stream) == 0
            if len(evs) == 3:
                evs[1].record(stream)
            assert lib.ref_attn_fwd(bf, q.data_ptr(), k.data_ptr(), v.data_ptr(), packed.data_ptr(),
                                    out.data_ptr(), lse.data_ptr(), B, H, N, D, 1.0 / math.sqrt(D), 0,
                                    stream.cuda_stream) == 0
            evs[-1].record(stream)

        n = max(5, min(args.steps, 50))
        for _ in range(max(args.warmup, 3)):
            flush()
            step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
        st = [s[0] for s in time_steps(step, n, flush, stream, marks=1)]
        sp = time_steps(step, n, flush, stream, marks=2)
        attn_mean = statistics.fmean([s[1] for s in sp])
        ev2 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        b2b = back_to_back_ms(lambda: step(ev2), stream)
        rl = attn_roofline(name, B, H, N, D, m, attn_mean, peaks)
        results[name] = {"step_ms_p50": p50(st), "back_to_back_ms_mean": b2b, "pack_ms_p50": p50([s[0] for s in sp]),
                         "attn_ms_p50": p50([s[1] for s in sp]), "attn_ms_mean": attn_mean,
                         "tflops_dense_equiv": workloads.dense_flops(B, H, N, D) / (p50(st) * 1e-3) / 1e12,
                         "roofline_frac": rl["frac"], "bound": rl["bound"], "steps": n}
        del q, k, v, m, packed, out, lse
        torch.cuda.empty_cache()
    c = results[args.config]
    cfg = workloads.CONFIGS[args.config]
    line = {"impl": "reference_cuda", "metric": METRIC,
            "value": workloads.dense_flops(cfg["B"], cfg["H"], cfg["N"], cfg["D"]) / (c["step_ms_p50"] * 1e-3) / 1e12,
            "unit": UNIT, "n_gpus": 1, "ms_per_step": c["step_ms_p50"], "higher_is_better": True,
            "config": workload_config(args.config, 1, args.config != "c5"),
            "kernels": "reference csrc/sparse_attention.cu pack_mask_kernel + sparse_attn_fwd_kernel<T>, sm_100a",
            "configs": results, "peaks": peaks}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm


def run_ours(args):
    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 under torchrun")
    from python import sparse_attention, sparse_attn_cuda, workloads
    from python.sharding import shard_range

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = workloads.CONFIGS[args.config]
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    weak = args.config != "c5"
    if weak:
        q, k, v, m = workloads.make_inputs(args.config, seed=args.seed + rank, device=dev)
    else:
        lo, hi = shard_range(B * H, world, rank)
        q, k, v, m = workloads.make_inputs(args.config, seed=args.seed, device=dev, heads=(lo, hi))
    lb, lh = q.shape[0], q.shape[1]
    flush = Flusher(dev)
    step = ForwardStep(q, k, v, m)
    stream = step.stream
    sampler = ClockSampler(dev)

    # correctness guard: the bench path equals the public API
    ref_out = sparse_attention(q, k, v, m)
    assert torch.equal(step(), ref_out)
    for _ in range(args.warmup):
        flush()
        step()
    sparse_attn_cuda.device_status()

    # ---- headline: exactly K timed steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    t_wall = time.perf_counter()
    for i in range(args.steps):
        flush()
        step(evs[i])
    torch.cuda.synchronize(dev)
    t_end = time.perf_counter()
    sampler.mark("timed", t_wall, t_end)
    sampler.stop()  # the clocks are reported for the timed steps above
    wall = t_end - t_wall
    if world > 1:
        torch.distributed.barrier()
    sparse_attn_cuda.device_status()
    step_ms = [e[0].elapsed_time(e[1]) for e in evs]

    # The two kernels timed apart, in a second pass of the same steps.
    split = time_steps(step, min(args.steps, 500), flush, stream, marks=2)
    # The reference's own timing of the same call: 50 back to back, no flush, mean.
    b2b_ms = max_over_ranks([back_to_back_ms(step, stream)], dev, world)[0]
    pack_ms = [s[0] for s in split]
    attn_ms = [s[1] for s in split]
    p50_step, mean_step, p50_attn, mean_attn, p50_pack, mean_pack = max_over_ranks(
        [p50(step_ms), statistics.fmean(step_ms), p50(attn_ms), statistics.fmean(attn_ms), p50(pack_ms),
         statistics.fmean(pack_ms)], dev, world)
    # The same steps after a memset-only flush (dirty L2 lines the packer must write back), for comparison.
    dirty = time_steps(step, min(args.steps, 100), flush, stream, marks=2, dirty=True)
    dirty_step_pack = max_over_ranks([p50([s[0] + s[1] for s in dirty]), p50([s[0] for s in dirty])], dev, world)

    # ---- optional NVLink gather of the output shards (timed separately; not part of a step)
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
        gather_ms = max_over_ranks([g0.elapsed_time(g1) / 10], dev, world)[0]
        del gathered

    # ---- end to end through the public API from pinned host memory:
    # sparse_attention_from_host (python/streaming.py) copies the inputs in,
    # computes and reads the output back, slice by slice so that PCIe carries
    # both directions at once; `plain` is the unsliced sequence (all copies
    # in, sparse_attention(), the copy back) for comparison.
    e2e = None
    if args.e2e_steps > 0:
        from python.streaming import sparse_attention_from_host

        hq, hk, hv, hm = (x.cpu().pin_memory() for x in (q, k, v, m))
        dq, dk, dv, dm = (torch.empty_like(x) for x in (q, k, v, m))
        hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()

        def streamed():
            sparse_attention_from_host(hq, hk, hv, hm, out=hout)

        def plain():
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            dm.copy_(hm, non_blocking=True)
            o = sparse_attention(dq, dk, dv, dm)
            hout.copy_(o, non_blocking=True)

        def e2e_p50(fn):
            e_times = []
            for i in range(args.e2e_steps + 3):
                flush()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn()
                b.record(stream)
                b.synchronize()
                if i >= 3:
                    e_times.append(a.elapsed_time(b))
            assert torch.equal(hout, ref_out.cpu())
            return max_over_ranks([p50(e_times)], dev, world)[0]

        et = e2e_p50(streamed)
        et_plain = e2e_p50(plain)
        flops_all = workloads.dense_flops(lb, lh, N, D) * (world if weak else 1)
        e2e = {"value": flops_all / (et * 1e-3) / 1e12, "unit": UNIT, "p50_ms": et,
               "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in (hq, hk, hv, hm)),
               "d2h_bytes_per_step": hout.numel() * hout.element_size(),
               "api": "sparse_attention_from_host (pinned host q/k/v/mask in, output back, sliced)",
               "plain": {"value": flops_all / (et_plain * 1e-3) / 1e12, "p50_ms": et_plain,
                         "api": "copies in, sparse_attention(), copy back"}}
        del hq, hk, hv, hm, dq, dk, dv, dm, hout

    peaks = load_peaks()
    blocks = {}
    if not args.no_blocks:
        del q, k, v, m, ref_out
        step = None
        torch.cuda.empty_cache()
        blocks["strong_c5"] = strong_c5_block(args, dev, flush, rank, world, peaks)
        if world == 1:
            blocks["configs"] = configs_block(args, dev, flush, peaks, blocks["strong_c5"])
            blocks["backward"] = backward_block(args, dev, flush, peaks)
            blocks["sweep"] = sweep_block(args, dev, flush, peaks)

    # ---- CPU baseline (the reference's CPU path) on rank 0 at N=1 only
    cpu_baseline = None
    if world == 1 and not args.no_cpu_baseline and args.config != "c5":
        t, threads, shape, reps = time_cpu(args.config, args.seed, args.cpu_seconds)
        b_, h_, n_, d_ = shape
        cpu_baseline = {"value": workloads.dense_flops(b_, h_, n_, d_) / t / 1e12, "unit": UNIT, "cores": threads,
                        "kind": "port", "ms": t * 1e3, "sample": cpu_sample_text(args.config, b_, h_, reps)}

    clocks = sampler.report("timed")
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0

    from python import workloads as wl

    rl = attn_roofline(args.config, lb, lh, N, D, step_mask_for_roofline(args, dev, rank, world), mean_attn, peaks)
    attn_kernel = "attn_fwd_chain_kernel"
    p_bytes = wl.pack_bytes(lb, lh, N)
    flops_step = wl.dense_flops(lb, lh, N, D)
    value = flops_step * (world if weak else 1) / (p50_step * 1e-3) / 1e12
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
        "scaling": "weak" if weak else "strong",
        "vs_baseline": None,
        "dtype": {torch.float16: "fp16", torch.bfloat16: "bf16"}[cfg["dtype"]],
        "data": "synthetic (seeded N(0,1) q/k/v, seeded masks per the workload recipe)",
        "config": workload_config(args.config, world, weak),
        "roofline": {"bound": "hbm", "achieved": rl["achieved_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": rl["hbm_frac"], "traffic": load_traffic(attn_kernel, args.config),
                     "kernel": attn_kernel, "algorithmic_bytes_per_launch": rl["algorithmic_bytes_per_launch"],
                     "avg_launch_ms": mean_attn, "peak_source": peaks["source"],
                     "roofline_bound": rl["bound"], "roofline_frac": rl["frac"]},
        "roofline_tensor": {"achieved": rl["achieved_tflops"], "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                            "frac": rl["tensor_frac"], "live_tile_fraction": rl["live_tile_fraction"],
                            "tile": rl["tile"]},
        "pack_roofline": {"achieved": p_bytes / (mean_pack * 1e-3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": p_bytes / (mean_pack * 1e-3) / 1e9 / peaks["hbm_gbs"],
                          "algorithmic_bytes_per_launch": p_bytes, "avg_launch_ms": mean_pack},
        "dirty_l2_flush": {"step_ms_p50": dirty_step_pack[0], "pack_ms_p50": dirty_step_pack[1],
                           "note": "memset-only flush: the packer also writes back the flush's dirty L2 lines"},
        "clocks": clocks,
        "gpu_launches": 2 * args.steps,
        "split_pass_steps": len(split),
        "back_to_back_ms_mean": b2b_ms,
        "timed_wall_s": wall,
    }
    if gather_ms is not None:
        line["gather_ms"] = gather_ms
    if e2e is not None:
        line["e2e"] = e2e
    if cpu_baseline is not None:
        line["cpu_baseline"] = cpu_baseline
    line.update(blocks)
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def step_mask_for_roofline(args, dev, rank, world):
    """The headline workload's mask on this rank (regenerated: the live-tile
    fraction is a property of the mask only)."""
    from python import workloads
    from python.sharding import shard_range

    cfg = workloads.CONFIGS[args.config]
    if args.config != "c5":
        return workloads.make_inputs(args.config, seed=args.seed + rank, device=dev)[3]
    lo, hi = shard_range(cfg["B"] * cfg["H"], world, rank)
    return workloads.make_inputs(args.config, seed=args.seed, device=dev, heads=(lo, hi))[3]


def strong_c5_block(args, dev, flush, rank, world, peaks):
    """c5 split by batch*head over the ranks; max-over-ranks p50 step and
    attention times.  t1 is one GPU running all of c5 in the same run (at
    N > 1 rank 0 times it alone while the other ranks wait)."""
    from python import workloads
    from python.sharding import shard_range

    cfg = workloads.CONFIGS["c5"]
    BH = cfg["B"] * cfg["H"]
    lo, hi = shard_range(BH, world, rank)
    steps = args.block_steps
    if world > 1:
        torch.distributed.barrier()
    r = measure_forward("c5", dev, flush, steps, args.seed, heads=(lo, hi))
    sp, sm, ap, am, pp = max_over_ranks([r["step_ms_p50"], r["step_ms_mean"], r["attn_ms_p50"], r["attn_ms_mean"],
                                         r["pack_ms_p50"]], dev, world)
    del r
    torch.cuda.empty_cache()
    t1 = None
    if world == 1:
        t1 = (sp, ap)
    else:
        torch.distributed.barrier()
        if rank == 0:
            r1 = measure_forward("c5", dev, flush, steps, args.seed)
            t1 = (r1["step_ms_p50"], r1["attn_ms_p50"])
            del r1
            torch.cuda.empty_cache()
        torch.distributed.barrier()
    if rank != 0:
        return None
    flops = workloads.dense_flops(cfg["B"], cfg["H"], cfg["N"], cfg["D"])
    return {"workload": f"c5: {workloads.describe('c5')} split over {world} rank(s) by batch*head",
            "n_gpus": world, "heads_per_rank_max": shard_range(BH, world, 0)[1], "steps": steps,
            "step_ms_p50": sp, "step_ms_mean": sm, "attn_ms_p50": ap, "attn_ms_mean": am, "pack_ms_p50": pp,
            "tflops_dense_equiv": flops / (sp * 1e-3) / 1e12,
            "t1_step_ms_p50": t1[0], "t1_attn_ms_p50": t1[1],
            "efficiency_step": t1[0] / (world * sp), "efficiency_attn": t1[1] / (world * ap),
            "timing": "per-rank CUDA events, p50, max over ranks; t1 = one GPU running all of c5 in this run"}


def configs_block(args, dev, flush, peaks, c5):
    """Every workload on one GPU under the same flush: step, pack and
    attention times and the attention kernel's roofline figures."""
    from python import workloads

    out = {}
    for name in ("c1", "c2", "c3", "c4", "c5"):
        r = measure_forward(name, dev, flush, args.block_steps, args.seed)
        q, m = r["q"], r["m"]
        B, H, N, D = q.shape
        rl = attn_roofline(name, B, H, N, D, m, r["attn_ms_mean"], peaks)
        out[name] = {"workload": workloads.describe(name), "step_ms_p50": r["step_ms_p50"],
                     "attn_ms_p50": r["attn_ms_p50"], "attn_ms_mean": r["attn_ms_mean"],
                     "pack_ms_p50": r["pack_ms_p50"],
                     "tflops_dense_equiv": workloads.dense_flops(B, H, N, D) / (r["step_ms_p50"] * 1e-3) / 1e12,
                     "bound": rl["bound"], "frac": rl["frac"], "hbm_frac": rl["hbm_frac"],
                     "tensor_frac": rl["tensor_frac"], "hbm_bound_us": rl["hbm_bound_us"],
                     "mma_bound_us": rl["mma_bound_us"], "live_tile_fraction": rl["live_tile_fraction"],
                     "tile": rl["tile"], "live_tile_fraction_128x64": rl["live_tile_fraction_128x64"],
                     "steps": args.block_steps}
        del r, q, m
        torch.cuda.empty_cache()
    return out


def sweep_block(args, dev, flush, peaks):
    """The reference's own performance sweep (run.py:483-540) on this library:
    sequence-length scaling (B chosen by N) and batch scaling at N = 512,
    H12 D64 fp16, prefix_random masks (python/workloads.py).  Per shape the
    step (pack + attention) p50, dense-equivalent TFLOPS, and the attention
    kernel's roofline fraction, under the same flush as every other block."""
    from python import workloads

    out = []
    for label, cfg in workloads.sweep_shapes():
        r = measure_forward(cfg, dev, flush, args.block_steps, args.seed)
        q, m = r["q"], r["m"]
        B, H, N, D = q.shape
        rl = attn_roofline(label, B, H, N, D, m, r["attn_ms_mean"], peaks)
        density = float(m.sum(dtype=torch.int64)) / m.numel()
        out.append({"shape": label, "B": B, "H": H, "N": N, "D": D, "density": density,
                    "step_ms_p50": r["step_ms_p50"], "attn_ms_p50": r["attn_ms_p50"],
                    "pack_ms_p50": r["pack_ms_p50"],
                    "tflops_dense_equiv": workloads.dense_flops(B, H, N, D) / (r["step_ms_p50"] * 1e-3) / 1e12,
                    "seq_per_s": B / (r["step_ms_p50"] * 1e-3), "bound": rl["bound"], "frac": rl["frac"],
                    "live_tile_fraction": rl["live_tile_fraction"], "steps": args.block_steps})
        del r, q, m
        torch.cuda.empty_cache()
    return out


def backward_block(args, dev, flush, peaks, name="c1"):
    r = measure_backward(name, dev, flush, args.block_steps, args.seed, peaks)
    return {k: v for k, v in r.items() if k not in ("clocks",)}


def measure_backward(name, dev, flush, steps, seed, peaks, warmup=3):
    """The backward kernels (sparse_attn_cuda.backward) on workload `name`."""
    from python import pack_mask, sparse_attn_cuda, workloads

    cfg = workloads.CONFIGS[name]
    B, H, N, D = cfg["B"], cfg["H"], cfg["N"], cfg["D"]
    q, k, v, m = workloads.make_inputs(name, seed=seed, device=dev)
    g = torch.Generator(device=dev).manual_seed(seed + 7)
    dout = torch.randn(q.shape, generator=g, device=dev).to(q.dtype)
    scale = 1.0 / math.sqrt(D)
    packed = pack_mask(m)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=dev, dtype=torch.float32)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, scale, True)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    stream = torch.cuda.current_stream(dev)

    def step(evs):
        evs[0].record(stream)
        sparse_attn_cuda.backward(dout, q, k, v, out, lse, packed, dq, dk, dv, scale)
        evs[1].record(stream)

    for _ in range(warmup):
        flush()
        step([torch.cuda.Event(enable_timing=True) for _ in range(2)])
    ms = [s[0] for s in time_steps(step, steps, flush, stream, marks=1)]
    sparse_attn_cuda.device_status()
    t = p50(ms)
    flops = workloads.backward_flops(B, H, N, D)
    nbytes = workloads.backward_bytes(B, H, N, D)
    live = workloads.live_tile_fraction(m, 128, 128)
    mma_flops = flops * live  # the kernel's five products run on live 128x128 tile pairs only
    return {"workload": f"{name}: {workloads.describe(name)}", "ms_p50": t, "steps": steps,
            "tflops_dense_equiv": flops / (t * 1e-3) / 1e12,
            "hbm_frac": nbytes / (t * 1e-3) / 1e9 / peaks["hbm_gbs"], "algorithmic_bytes_per_step": nbytes,
            "tensor_frac": mma_flops / (t * 1e-3) / 1e12 / peaks["bf16_tflops"], "live_tile_fraction": live,
            "gpu_launches_per_step": 3}


def run_backward(args):
    """One GPU: the backward (dq, dk, dv from dout and the forward's out and
    lse) on the workload, inputs resident in HBM, L2 flushed before every
    step.  Prints one JSON line in the forward's format."""
    rank, world, local = dist_env()
    if world != 1 or args.gpus != 1:
        raise SystemExit("--pass backward runs on one GPU")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    flush = Flusher(dev)
    peaks = load_peaks()
    sampler = ClockSampler(dev)
    t0 = time.perf_counter()
    r = measure_backward(args.config, dev, flush, args.steps, args.seed, peaks, warmup=args.warmup)
    sampler.mark("timed", t0, time.perf_counter())
    line = {
        "metric": "backward dense-equiv TFLOPS (10*B*H*N^2*D / p50 step)",
        "value": r["tflops_dense_equiv"],
        "unit": "TFLOPS",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": r["ms_p50"],
        "higher_is_better": True,
        "config": {"workload": r["workload"], "pass": "backward", "l2": L2_NOTE},
        "backward": r,
        "clocks": sampler.report("timed"),
        "gpu_launches": 3 * args.steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "reference_cuda":
        return run_reference_cuda(args)
    if args.which == "backward":
        return run_backward(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
