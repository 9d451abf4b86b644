#!/usr/bin/env python3
"""Benchmark of UserOptimizedTransformer.forward on B200s (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

Metric (BASELINE): forward latency and tokens/s per config, MFU against the
B200 dense tensor peak. A "step" is one forward pass over one batch of
synthetic input (x ~ N(0,1), default-initialised weights, fp32 model,
fp16 tensor-core compute). The headline workload is c3 (B8 S2048 D1024 H16
F4096 L12): the first BASELINE config that is tensor-core bound and
batch-sharded; the other configs are reported under "per_config" at N=1.

Timing: W untimed warm-up steps (the first captures the CUDA graph), then
exactly K steps, each bracketed by CUDA events on the launching stream, with
a 256 MB L2 flush between steps (outside the events); a barrier and a device
synchronise on both sides; the max over ranks. With N>1 every rank runs its
own batch of the config (data parallel, no collective on the data path:
"scaling": "weak"), and value = total tokens of all ranks / max time.

--impl reference times the reference algorithm on the host CPU (the oracle's
restatement of BaselineTransformer, all host threads) on a bounded exact slice
of the same workload: one batch element through every layer.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from transformer_optimization_b200 import NAMED_CONFIGS, UserOptimizedTransformer, count_dense_flops  # noqa: E402
from transformer_optimization_b200 import kernels as K  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) per projection launch of the c3 forward, mean of
# the four projections of a layer, from one ncu capture of each shape (the
# capture summaries are kept with the profiles)
C3_GEMM_DRAM_BYTES_PER_LAUNCH = 150.9e6
L2_FLUSH_BYTES = 256 << 20


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def algo_bytes_per_gemm(cfg, x_bytes=4):
    """Mean algorithmic HBM bytes of the four projections of one layer:
    16-bit A and W read, 16-bit C written (QKV, FFN in), or the residual x
    (x_bytes per element: 4 for the fp32 model, 2 for fp16/bf16 models) read
    and written around the product (the two residual projections)."""
    m, d, f = cfg.batch_size * cfg.seq_len, cfg.d_model, cfg.ffn_dim
    qkv = 2 * (m * d + 3 * d * d + 3 * m * d)
    ffn_in = 2 * (m * d + f * d + m * f)
    out_proj = 2 * (m * d + d * d) + 2 * x_bytes * m * d
    ffn_out = 2 * (m * f + d * f) + 2 * x_bytes * m * d
    return (qkv + ffn_in + out_proj + ffn_out) / 4


def cfg_dict(cfg):
    return {"B": cfg.batch_size, "S": cfg.seq_len, "D": cfg.d_model, "H": cfg.num_heads,
            "F": cfg.ffn_dim, "L": cfg.num_layers, "causal": cfg.causal}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [r for r in rows if r[2] > 300.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


# ---------------------------------------------------------------- helpers
MODEL_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def build_model(cfg, device, dtype=torch.float32):
    torch.manual_seed(0)
    with torch.device(device):
        model = UserOptimizedTransformer(cfg)
    return model.to(dtype).eval()


def flush_l2(buf):
    buf.zero_()


def time_steps(fn, steps, flush_buf):
    """Per-step CUDA events on the current stream; L2 flushed between steps
    outside the events. Returns the list of step times in ms."""
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_l2(flush_buf)
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def e2e_pipelined(model, x_host, y_host, steps, device):
    """`steps` forward passes through the public module, each with its own
    host-to-device copy of the pinned input and device-to-host copy of the
    output, as a serving loop runs them: the copies go on two copy streams
    (double-buffered device input), so step i+1's upload and step i-1's
    download overlap step i's forward. One CUDA-event pair brackets the whole
    sequence, first upload to last download. Returns the total in ms."""
    comp = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    xd = [torch.empty(x_host.shape, dtype=x_host.dtype, device=device) for _ in range(2)]
    ev = lambda: torch.cuda.Event()  # noqa: E731
    fwd_done = [None] * steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(comp)
    up.wait_event(start)
    down.wait_event(start)
    for i in range(steps):
        b = i % 2
        with torch.cuda.stream(up):
            if i >= 2:
                up.wait_event(fwd_done[i - 2])  # the forward that read this buffer is done
            xd[b].copy_(x_host, non_blocking=True)
            uploaded = ev()
            uploaded.record(up)
        comp.wait_event(uploaded)
        y = model(xd[b])
        fwd_done[i] = ev()
        fwd_done[i].record(comp)
        with torch.cuda.stream(down):
            down.wait_event(fwd_done[i])
            y_host.copy_(y, non_blocking=True)
            y.record_stream(down)
    comp.wait_stream(down)
    end.record(comp)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def kernel_profile(model, x):
    """One instrumented eager forward: CUDA events around every launch of the
    GEMM, attention and LayerNorm kernels (on the launching stream).
    Returns {kernel: (launches, total_ms, algorithmic units)}."""
    cfg = model.config
    rec = {"gemm": [], "flash": [], "ln": []}
    orig = (K.linear, K.flash_attention, K.ln_residual, K.linear_residual)

    def wrap(name, f, units):
        def g(*a, **kw):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            r = f(*a, **kw)
            e.record()
            rec[name].append((s, e, units(*a, **kw)))
            return r
        return g

    def gemm_flops(a, w, b, *args, **kw):
        # algorithmic flops of the projection (split weights do twice the
        # tensor work for the same product; counted once)
        return 2.0 * (a.numel() // a.shape[-1]) * a.shape[-1] * w.shape[0]

    def flash_flops(q, k, v, heads, scale, **kw):
        bsz, sq, dq = q.shape
        sk = k.shape[1]
        return 4.0 * bsz * sq * sk * dq  # dense count (run_bench.py convention)

    def ln_bytes(x, delta, w, b, eps, valid=None, **kw):
        n, xs = x.numel(), x.element_size()
        by = n * xs + (n * 2 if delta is not None else 0)
        by += n * xs if kw.get("write_x") else 0
        by += n * (4 if kw.get("out_dtype") == torch.float32 else 2)
        return float(by)

    K.linear = wrap("gemm", orig[0], gemm_flops)
    K.flash_attention = wrap("flash", orig[1], flash_flops)
    K.ln_residual = wrap("ln", orig[2], ln_bytes)
    K.linear_residual = wrap("gemm", orig[3], gemm_flops)
    try:
        model.use_cuda_graphs = False
        with torch.inference_mode():
            # the first eager pass warms the allocator's pools for the eager
            # buffers (a cudaMalloc between two events would be timed)
            model(x)
            torch.cuda.synchronize()
            for lst in rec.values():
                lst.clear()
            # hold the GPU for ~0.1 s so the host enqueues the whole forward
            # ahead of it: the launches then run back to back and each event
            # pair brackets device time only, not the host's launch latency
            torch.cuda._sleep(200_000_000)
            model(x)
        torch.cuda.synchronize()
    finally:
        K.linear, K.flash_attention, K.ln_residual, K.linear_residual = orig
        model.use_cuda_graphs = True
    out = {}
    for name, lst in rec.items():
        ms = sum(s.elapsed_time(e) for s, e, _ in lst)
        out[name] = (len(lst), ms, sum(u for _, _, u in lst))
    return out


def cpu_reference_sample(cfg, threads, min_seconds=8.0, max_reps=3):
    """The oracle's fp32 eager forward (reference BaselineTransformer
    arithmetic) on the host CPU: one batch element through every layer, an
    exact slice of the workload (per-token cost is the same for every batch
    element). Returns (tokens/s, sample description, ms per slice)."""
    from oracle import reference_model as om
    torch.set_num_threads(threads)
    sub = type(cfg)(1, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers, cfg.causal)
    p = om.init_params(sub, 0)
    x = torch.randn(1, cfg.seq_len, cfg.d_model)
    qt = 1024 if cfg.seq_len > 8192 else None
    layers = sub.num_layers
    # very long slices: time a prefix of the layers and scale (cost is linear in layers)
    times = []
    t_start = time.perf_counter()
    with torch.inference_mode():
        while len(times) < max_reps:
            t0 = time.perf_counter()
            om.forward(p, sub, x, query_tile=qt, ffn_row_chunk=4096 if qt else None, layers=layers)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > min_seconds:
                break
    t = statistics.median(times)
    per_forward = t * cfg.num_layers / layers
    return (cfg.seq_len / per_forward,
            f"1 of {cfg.batch_size} batch elements ({cfg.seq_len} tokens) x {layers} of {cfg.num_layers} layers, "
            f"median of {len(times)}", per_forward * 1000.0)


# ---------------------------------------------------------------- arms
def run_reference(args, cfg, rank):
    threads = os.cpu_count() or 1
    if rank != 0:
        return
    tok_s, sample, _ = cpu_reference_sample(cfg, threads)
    line = {
        "impl": "reference", "metric": f"forward tokens/s ({args.config})", "value": tok_s, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": cfg.batch_size * cfg.seq_len / tok_s * 1000.0, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, **cfg_dict(cfg), "parallelism": "host cpu"},
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measure_config(cfg, device, steps, warmup, flush_buf, dtype=torch.float32):
    model = build_model(cfg, device, dtype)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, device=device).to(dtype)
    with torch.inference_mode():
        for _ in range(warmup):
            model(x)
        torch.cuda.synchronize()
        ts = time_steps(lambda: model(x), steps, flush_buf)
    del model
    return ts


def run_ours(args, cfg, rank, world, local_rank):
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist
    peaks, peak_src = load_peaks()
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    mdt = MODEL_DTYPES[args.model_dtype]
    model = build_model(cfg, device, mdt)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, device=device).to(mdt)
    tokens = cfg.batch_size * cfg.seq_len
    with torch.inference_mode():
        for _ in range(max(args.warmup, 3)):
            model(x)
    torch.cuda.synchronize()

    # ---- device-timed steps (inputs resident in HBM) ----
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    smi_id = vis.split(",")[local_rank].strip() if vis else str(local_rank)
    with ClockSampler(smi_id) as clk:
        with torch.inference_mode():
            ts = time_steps(lambda: model(x), args.steps, flush_buf)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    total_ms = sum(ts)
    if dist is not None:
        t = torch.tensor([total_ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * tokens / (ms_per_step / 1000.0)

    # ---- end to end through the public module: pinned host in, host out ----
    x_host = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model).to(mdt).pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    with torch.inference_mode():
        e2e_pipelined(model, x_host, y_host, 2, device)  # warm-up (allocations, streams)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e_total = e2e_pipelined(model, x_host, y_host, args.steps, device)
    if dist is not None:
        t = torch.tensor([e_total], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_total = float(t.item())
        dist.barrier()
    e2e_value = world * tokens / (e_total / args.steps / 1000.0)

    # ---- per-kernel roofline from an instrumented eager forward ----
    prof = kernel_profile(model, x)
    flops = count_dense_flops(cfg)
    tensor_peak = peaks["bf16_tflops"]
    # kernels timed inside a long step run at the sustained (power-capped) clock
    sustained = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    n_g, ms_g, fl_g = prof["gemm"]
    n_f, ms_f, fl_f = prof["flash"]
    n_l, ms_l, by_l = prof["ln"]
    gemm_tflops = fl_g / (ms_g / 1e3) / 1e12
    flash_tflops = fl_f / (ms_f / 1e3) / 1e12
    ln_gbs = by_l / (ms_l / 1e3) / 1e9
    launches_per_step = n_g + n_f + n_l

    line = {
        "metric": f"forward tokens/s ({args.config})", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if mdt == torch.bfloat16 else "f16",
        "data": "synthetic",
        "config": {"workload": args.config, **cfg_dict(cfg), "global_batch": cfg.batch_size * world,
                   "parallelism": f"dp{world}", "l2": "flushed between steps (256 MB write)",
                   "weights": "default init, seed 0", "cuda_graph": True, "model_dtype": args.model_dtype},
        "mfu": flops / (ms_per_step / 1e3) / (tensor_peak * 1e12),
        "latency_ms": ms_per_step, "latency_ms_median": statistics.median(ts),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                "d2h_bytes_per_step": y_host.numel() * y_host.element_size(), "ms_per_step": e_total / args.steps,
                "copies": "pinned H2D and D2H every step on two copy streams, overlapping the neighbouring "
                          "steps' forwards; one event pair from the first upload to the last download"},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": {"bound": "tensor", "kernel": "gemm_f16_tcgen05", "achieved": gemm_tflops,
                     "peak": sustained, "unit": "TFLOP/s", "frac": gemm_tflops / sustained,
                     "peak_source": f"bf16_tflops_sustained ({peak_src}): the GEMMs are timed inside the step",
                     "traffic": (C3_GEMM_DRAM_BYTES_PER_LAUNCH
                                 if args.config == "c3" and mdt == torch.float32 else None),
                     "traffic_unit": "bytes per launch (ncu dram read+write)",
                     "algorithmic_bytes_per_launch": algo_bytes_per_gemm(cfg, x.element_size()),
                     "launches_per_step": n_g, "gemm_share_of_step": ms_g / ms_per_step},
        "kernels": {
            "flash_fwd_tcgen05": {"launches": n_f, "ms": ms_f, "tflops": flash_tflops,
                                  "frac": flash_tflops / sustained},
            "ln_residual": {"launches": n_l, "ms": ms_l, "gbs": ln_gbs, "frac": ln_gbs / peaks["hbm_gbs"]},
            "gemm_f16_tcgen05": {"launches": n_g, "ms": ms_g, "tflops": gemm_tflops},
        },
        "clocks": clk.summary(),
    }

    del model, x
    torch.cuda.empty_cache()
    if world == 1 and not args.no_extra:
        # other BASELINE configs at N=1 (device-timed latency; same protocol)
        per = {}
        for name in ("c1", "c2", "c3", "c4", "c5"):
            c = NAMED_CONFIGS[name]
            if name == args.config:
                ts_c = ts
            else:
                ts_c = measure_config(c, device, max(3, args.steps // 4), 3, flush_buf, mdt)
            lat = statistics.median(ts_c)
            per[name] = {"latency_ms": lat, "tokens_per_s": c.batch_size * c.seq_len / (lat / 1e3),
                         "mfu": count_dense_flops(c) / (lat / 1e3) / (tensor_peak * 1e12)}
        line["per_config"] = per
        threads = os.cpu_count() or 1
        tok_s, sample, _ = cpu_reference_sample(cfg, threads)
        line["cpu_baseline"] = {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
                                "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_cp(args, cfg, rank, world, local_rank):
    """Context-parallel forward of one long sequence over `world` GPUs (ring
    attention over NCCL P2P). Strong scaling: the same sequence is split."""
    import torch.distributed as dist

    from transformer_optimization_b200.context_parallel import ContextParallelTransformer, shard_bounds
    device = torch.device("cuda", local_rank)
    peaks, peak_src = load_peaks()
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    model = build_model(cfg, device)  # same seed on every rank: identical weights
    bounds = shard_bounds(cfg.seq_len, world)
    st, n = bounds[rank]
    x_local = torch.randn(cfg.batch_size, n, cfg.d_model, device=device)
    cp = ContextParallelTransformer(model)
    with torch.inference_mode():
        for _ in range(max(args.warmup, 3)):
            cp.forward(x_local, bounds=bounds)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    smi_id = vis.split(",")[local_rank].strip() if vis else str(local_rank)
    with ClockSampler(smi_id) as clk:
        with torch.inference_mode():
            ts = time_steps(lambda: cp.forward(x_local, bounds=bounds), args.steps, flush_buf)
    torch.cuda.synchronize()
    dist.barrier()
    t = torch.tensor([sum(ts)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    tokens = cfg.batch_size * cfg.seq_len
    value = tokens / (ms_per_step / 1e3)

    x_host = torch.randn(cfg.batch_size, n, cfg.d_model).pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()

    def e2e_step():
        y = cp.forward(x_host.to(device, non_blocking=True), bounds=bounds)
        y_host.copy_(y, non_blocking=True)

    with torch.inference_mode():
        e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        e_ts = time_steps(e2e_step, args.steps, flush_buf)
    t = torch.tensor([sum(e_ts)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e_ms = float(t.item()) / args.steps
    dist.barrier()
    flops = count_dense_flops(cfg)
    launches = cfg.num_layers * (6 + world + (world - 1)) + 1
    line = {
        "metric": f"forward tokens/s ({args.config})", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": args.config, **cfg_dict(cfg), "global_batch": cfg.batch_size,
                   "parallelism": f"cp{world}", "shard_tokens": n, "l2": "flushed between steps (256 MB write)",
                   "weights": "default init, seed 0", "cuda_graph": False},
        "mfu": flops / (ms_per_step / 1e3) / (peaks["bf16_tflops"] * 1e12 * world),
        "latency_ms": ms_per_step,
        "e2e": {"value": tokens / (e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": x_host.numel() * 4 * world, "d2h_bytes_per_step": y_host.numel() * 4 * world,
                "ms_per_step": e_ms},
        "gpu_launches": launches * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[1])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", choices=sorted(NAMED_CONFIGS))
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-extra", action="store_true", help="skip per_config and cpu_baseline")
    ap.add_argument("--model-dtype", default="float32", choices=sorted(MODEL_DTYPES),
                    help="parameter and input dtype of the model (the BASELINE configs are float32)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = NAMED_CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"[bench] warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)

    if args.impl == "reference":
        run_reference(args, cfg, rank)
        return 0

    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if world > 1 and cfg.batch_size == 1:
            if args.model_dtype != "float32":
                raise SystemExit("context parallelism runs the float32 model")
            run_cp(args, cfg, rank, world, local_rank)  # one sequence: context parallel
        else:
            run_ours(args, cfg, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
