#!/usr/bin/env python3
"""Benchmark of UserOptimizedTransformer.forward on B200s (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]

Metric (BASELINE): forward latency and tokens/s per config, MFU against the
B200 dense tensor peak, at 1 GPU and at 2/4/8 GPUs where the config shards.
A "step" is one forward pass over one batch of synthetic input (x ~ N(0,1),
default-initialised weights under seed 0, fp32 model, fp16 tensor-core
compute with fp32 accumulation).

Headline: c3 (B8 S2048 D1024 H16 F4096 L12), the first BASELINE config that
is tensor-core bound, BATCH-SHARDED over the N ranks (data parallel, no
collective on the data path): rank r runs its B/N batch elements of the same
seeded input, and the line's value is the whole batch's tokens divided by
the slowest rank's time ("scaling": "strong"; the config is the same at
every N). Further keys on the same line:
  c5_cp    c5 (S = 100000) context parallel over the N ranks: ring attention
           over NCCL P2P, strong scaling, with the per-layer ring breakdown
           (flash blocks, merges, exposed exchange wait) from an
           instrumented forward;
  c4_dp    c4 (B32 S4096 D2048 L24) batch-sharded like the headline;
  weak     (N > 1) every rank runs the whole c3 batch (weak scaling);
  per_config  every BASELINE config's latency, tokens/s, MFU (c1, c2 are
           replicas-only and measured at N = 1);
  cpu_baseline (N = 1) the reference algorithm on the host CPU: a full c3
           forward (all 8 batch elements, all 12 layers), median of 3.

Timing: W untimed warm-up steps (the first captures the CUDA graph), then
exactly K steps, each bracketed by CUDA events on the launching stream, with
a 256 MB L2 flush between steps (outside the events); a barrier and a device
synchronise on both sides; the max over ranks. GPU clocks are sampled with
nvidia-smi every 50 ms and only samples inside timed windows are kept.

--impl reference times the reference algorithm on the host CPU (the oracle's
restatement of BaselineTransformer, all host threads); each of its W + K
steps is a bounded, exact sample of the workload: one batch element of c3
through all layers (per-token cost is the same for every batch element).
Under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import platform
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
_JSON_OUT = None  # the process's original stdout; everything else goes to stderr


def emit(line: dict) -> None:
    """Print the one JSON line on the original stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


# DRAM bytes (read + write) per projection launch of the c3 forward at one
# GPU (M = 16384 rows), mean of the four projections of a layer, from one ncu
# capture of each shape (the capture summaries are kept with the profiles)
C3_GEMM_DRAM_BYTES_PER_LAUNCH = 153.3e6
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


def algo_bytes_per_gemm(cfg, x_bytes=4, rows=None):
    """Mean algorithmic HBM bytes of the four projections of one layer:
    16-bit A and W read, 16-bit C written (QKV, FFN in), or the residual x
    (x_bytes per element: 4 for the fp32 model, 2 for fp16/bf16 models) read
    and written around the product (the two residual projections). rows:
    the rows one launch processes (default: the whole config's B*S)."""
    m = cfg.batch_size * cfg.seq_len if rows is None else rows
    d, f = cfg.d_model, cfg.ffn_dim
    qkv = 2 * (m * d + 3 * d * d + 3 * m * d)
    ffn_in = 2 * (m * d + f * d + m * f)
    out_proj = 2 * (m * d + d * d) + 2 * x_bytes * m * d
    ffn_out = 2 * (m * f + d * f) + 2 * x_bytes * m * d
    return (qkv + ffn_in + out_proj + ffn_out) / 4


def cfg_dict(cfg):
    return {"B": cfg.batch_size, "S": cfg.seq_len, "D": cfg.d_model, "H": cfg.num_heads,
            "F": cfg.ffn_dim, "L": cfg.num_layers, "causal": cfg.causal}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def shard_sizes(total: int, world: int):
    """Even split of `total` items over `world` ranks (the first ranks take
    one more): [(start, count)] per rank."""
    base, rem = divmod(total, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < rem else 0)
        out.append((start, n))
        start += n
    return out


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 50 ms) of SM clock and throttle reasons over
    the whole measurement; only samples inside the recorded timed windows
    (host wall clock around each device-timed region) are summarised."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: str):
        self.gpu = gpu_index
        self.proc = None
        self.out = ""
        self.windows = {}  # name -> [(t0, t1)] in epoch seconds

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""
            self.proc = None

    def window(self, name):
        sampler = self

        class _W:
            def __enter__(self_):
                self_.t0 = time.time()

            def __exit__(self_, *exc):
                sampler.windows.setdefault(name, []).append((self_.t0, time.time()))
        return _W()

    def _rows(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            parts = [s.strip() for s in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(parts[2]), float(parts[3]), float(parts[4]), parts[6:10]))
            except ValueError:
                continue
        return rows

    def summary(self, names=None):
        rows = self._rows()
        wins = [w for n, ws in self.windows.items() if names is None or n in names for w in ws]
        inside = [r for r in rows if any(t0 <= r[0] <= t1 for t0, t1 in wins)]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": max((r[2] for r in rows), default=None),
                    "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({self.NAMES[i] for r in inside for i, v in enumerate(r[4]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in rows),
                "reasons": reasons, "samples": len(inside), "power_w_median": statistics.median(r[3] for r in inside)}


# ---------------------------------------------------------------- helpers
MODEL_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def build_model(cfg, device, dtype=torch.float32):
    """Default-initialised weights under seed 0: identical on every rank."""
    torch.manual_seed(0)
    with torch.device(device):
        model = UserOptimizedTransformer(cfg)
    return model.to(dtype).eval()


def seeded_input(cfg, device, dtype, b0, nb):
    """Batch elements [b0, b0 + nb) of the config's seeded input (the same
    global tensor on every rank: seed 1 on the device generator)."""
    torch.manual_seed(1)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, device=device)
    return x[b0:b0 + nb].to(dtype).contiguous()


def time_steps(fn, steps, flush_buf):
    """Per-step CUDA events on the current stream; L2 flushed between steps
    outside the events. Returns the list of step times in ms."""
    stream = torch.cuda.current_stream()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush_buf.zero_()
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def max_over_ranks(v: float, dist, device) -> float:
    if dist is None:
        return v
    t = torch.tensor([v], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()


def e2e_serial(model_fn, x_host, y_host, steps, device, flush_buf):
    """`steps` forwards through the public API, each one serial: pinned
    host-to-device copy of the input, forward, device-to-host copy of the
    output, all on the current stream between one event pair (the
    per-forward latency a caller sees). Returns per-step ms."""
    xd = torch.empty(x_host.shape, dtype=x_host.dtype, device=device)

    def step():
        xd.copy_(x_host, non_blocking=True)
        y = model_fn(xd)
        y_host.copy_(y, non_blocking=True)
    return time_steps(step, steps, flush_buf)


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
    GEMM, attention and LayerNorm kernels (on the launching stream). The
    events serialise the launches, so a LayerNorm that overlaps its residual
    GEMM's tail in the graph (ln_ready) is timed here on its own.
    Returns {kernel: (launches, total_ms, algorithmic units)}."""
    rec = {"gemm": [], "flash": [], "ln": []}
    orig = (K.linear, K.flash_attention, K.ln_residual, K.linear_residual, K.linear_residual_ln, K.ln_ready)

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

    def ln_ready_bytes(x, w, b, eps, ready, valid=None, **kw):
        n = x.numel()
        return float(n * x.element_size() + n * (4 if kw.get("out_dtype") == torch.float32 else 2))

    K.linear = wrap("gemm", orig[0], gemm_flops)
    K.flash_attention = wrap("flash", orig[1], flash_flops)
    K.ln_residual = wrap("ln", orig[2], ln_bytes)
    K.linear_residual = wrap("gemm", orig[3], gemm_flops)
    K.linear_residual_ln = wrap("gemm", orig[4], gemm_flops)
    K.ln_ready = wrap("ln", orig[5], ln_ready_bytes)
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
        K.linear, K.flash_attention, K.ln_residual, K.linear_residual, K.linear_residual_ln, K.ln_ready = orig
        model.use_cuda_graphs = True
    out = {}
    for name, lst in rec.items():
        ms = sum(s.elapsed_time(e) for s, e, _ in lst)
        out[name] = (len(lst), ms, sum(u for _, _, u in lst))
    return out


def cpu_reference_forward(cfg, threads, batch_elems, reps, warmup=0):
    """The oracle's fp32 eager forward (reference BaselineTransformer
    arithmetic) on the host CPU over `batch_elems` batch elements of the
    config through every layer. Returns the per-repetition seconds."""
    from oracle import reference_model as om
    torch.set_num_threads(threads)
    sub = type(cfg)(batch_elems, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers, cfg.causal)
    p = om.init_params(sub, 0)
    x = torch.randn(batch_elems, cfg.seq_len, cfg.d_model)
    qt = 1024 if cfg.seq_len > 8192 else None
    times = []
    with torch.inference_mode():
        for i in range(warmup + reps):
            t0 = time.perf_counter()
            om.forward(p, sub, x, query_tile=qt, ffn_row_chunk=4096 if qt else None)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    return times


# ---------------------------------------------------------------- reference arm
def run_reference(args, cfg, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # each step: one batch element of the workload through every layer
    times = cpu_reference_forward(cfg, threads, 1, args.steps, warmup=args.warmup)
    ms = [t * 1e3 for t in times]
    tok = cfg.seq_len * len(times)
    tok_s = tok / sum(times)
    sample = (f"each step: 1 of {cfg.batch_size} batch elements ({cfg.seq_len} tokens) through all "
              f"{cfg.num_layers} layers; {args.warmup} warm-up + {args.steps} timed steps run")
    line = {
        "impl": "reference", "metric": f"forward tokens/s ({args.config})", "value": tok_s, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": statistics.mean(ms), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, **cfg_dict(cfg), "parallelism": "host cpu",
                   "step_tokens": cfg.seq_len},
        "latency_ms_full_forward_extrapolated": statistics.median(ms) * cfg.batch_size,
        "cpu_baseline": {"value": tok_s, "unit": "tokens/s", "cores": threads, "cpu_model": cpu_model(),
                         "kind": "port", "sample": sample, "extrapolated": False},
        "e2e": {"value": tok_s, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ---------------------------------------------------------------- our arm
class Ctx:
    def __init__(self, args, rank, world, local_rank, dist):
        self.args, self.rank, self.world, self.dist = args, rank, world, dist
        self.device = torch.device("cuda", local_rank)
        self.peaks, self.peak_src = load_peaks()
        self.flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=self.device)
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        self.smi_id = vis.split(",")[local_rank].strip() if vis else str(local_rank)
        self.clk = ClockSampler(self.smi_id)

    def mfu(self, cfg, ms):
        return count_dense_flops(cfg) / (ms / 1e3) / (self.peaks["bf16_tflops"] * 1e12 * self.world)


def measure_sharded(c: Ctx, cfg, steps, warmup, window, mdt=torch.float32, keep=False):
    """Batch-sharded forward of `cfg` over the ranks (strong scaling): max
    over ranks of the per-step time. Returns (summary dict, model, x) when
    `keep`, else (summary, None, None)."""
    if cfg.batch_size < c.world:
        raise SystemExit(f"{cfg.batch_size} batch elements cannot be sharded over {c.world} ranks")
    b0, nb = shard_sizes(cfg.batch_size, c.world)[c.rank]
    model = build_model(cfg, c.device, mdt)
    x = seeded_input(cfg, c.device, mdt, b0, nb)
    with torch.inference_mode():
        for _ in range(max(warmup, 3)):
            model(x)
    barrier(c.dist)
    with c.clk.window(window):
        with torch.inference_mode():
            ts = time_steps(lambda: model(x), steps, c.flush_buf)
    barrier(c.dist)
    ms = max_over_ranks(sum(ts) / steps, c.dist, c.device)
    med = max_over_ranks(statistics.median(ts), c.dist, c.device)
    tokens = cfg.batch_size * cfg.seq_len
    out = {"latency_ms": ms, "latency_ms_median": med, "tokens_per_s": tokens / (ms / 1e3),
           "mfu": c.mfu(cfg, ms), "steps": steps, "rank_batch": nb, "parallelism": f"dp{c.world}"}
    if keep:
        return out, model, x
    del model, x
    torch.cuda.empty_cache()
    return out, None, None


def ring_breakdown(cp, x_local, layout, layers):
    """One instrumented context-parallel forward: per-forward ms of the flash
    blocks, the merges and the exposed exchange waits (CUDA events on the
    compute stream), and the ring steps per layer."""
    tl = []
    cp.ring.timeline = tl
    try:
        with torch.inference_mode():
            cp.forward(x_local, layout=layout)
        torch.cuda.synchronize()
    finally:
        cp.ring.timeline = None
        cp.ring.backend.timeline = None
    tot = {"block": 0.0, "merge": 0.0, "wait": 0.0}
    for kind, s, e in tl:
        tot[kind] += s.elapsed_time(e)
    steps = sum(1 for kind, _, _ in tl if kind == "block")
    return {"flash_ms": tot["block"] - tot["merge"], "merge_ms": tot["merge"], "exposed_wait_ms": tot["wait"],
            "ring_steps_per_layer": steps // max(layers, 1)}


def measure_cp(c: Ctx, cfg, steps, warmup, window):
    """c5-style single-sequence config over the ranks: N = 1 the model's own
    forward; N > 1 context parallel (contiguous shards; zigzag when causal)."""
    from transformer_optimization_b200.context_parallel import (ContextParallelTransformer, contiguous_layout,
                                                                local_positions, zigzag_layout)
    model = build_model(cfg, c.device)
    tokens = cfg.batch_size * cfg.seq_len
    if c.world == 1:
        x = seeded_input(cfg, c.device, torch.float32, 0, cfg.batch_size)
        fn = model
        layout_kind = "single"
    else:
        layout_kind = "zigzag" if cfg.causal else "contiguous"
        layout = (zigzag_layout if cfg.causal else contiguous_layout)(cfg.seq_len, c.world)
        rows = local_positions(layout[c.rank]).to(c.device)
        x = seeded_input(cfg, c.device, torch.float32, 0, cfg.batch_size)[:, rows].contiguous()
        cp = ContextParallelTransformer(model)
        fn = lambda xx: cp.forward(xx, layout=layout)  # noqa: E731
    with torch.inference_mode():
        for _ in range(max(warmup, 2)):
            fn(x)
    barrier(c.dist)
    with c.clk.window(window):
        with torch.inference_mode():
            ts = time_steps(lambda: fn(x), steps, c.flush_buf)
    barrier(c.dist)
    ms = max_over_ranks(sum(ts) / steps, c.dist, c.device)
    out = {"latency_ms": ms, "latency_ms_median": max_over_ranks(statistics.median(ts), c.dist, c.device),
           "tokens_per_s": tokens / (ms / 1e3), "mfu": c.mfu(cfg, ms), "steps": steps,
           "parallelism": f"cp{c.world}", "layout": layout_kind, "nccl_ranks": c.world,
           "shard_tokens": int(x.shape[1])}
    # serial end to end: this rank's shard in from pinned host memory, out to it
    x_host = x.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    with torch.inference_mode():
        e2e_serial(fn, x_host, y_host, 1, c.device, c.flush_buf)
        barrier(c.dist)
        with c.clk.window(window):
            e_ts = e2e_serial(fn, x_host, y_host, steps, c.device, c.flush_buf)
    barrier(c.dist)
    e_ms = max_over_ranks(sum(e_ts) / steps, c.dist, c.device)
    out["e2e"] = {"value": tokens / (e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e_ms,
                  "h2d_bytes_per_step": x_host.numel() * 4 * c.world,
                  "d2h_bytes_per_step": y_host.numel() * 4 * c.world, "copies": "serial"}
    if c.world > 1:
        rb = ring_breakdown(cp, x, layout, cfg.num_layers)
        vals = torch.tensor([rb["flash_ms"], rb["merge_ms"], rb["exposed_wait_ms"]], device=c.device,
                            dtype=torch.float64)
        if c.dist is not None:
            c.dist.all_reduce(vals, op=c.dist.ReduceOp.MAX)
        rb.update(flash_ms=float(vals[0]), merge_ms=float(vals[1]), exposed_wait_ms=float(vals[2]),
                  kv_bytes_per_step=2 * int(x.shape[1]) * cfg.d_model * 2, note="max over ranks, one forward")
        out["ring"] = rb
    del model, x, fn
    if c.world > 1:
        del cp
    torch.cuda.empty_cache()
    return out


def run_ours(args, cfg, rank, world, local_rank):
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist
    c = Ctx(args, rank, world, local_rank, dist)
    mdt = MODEL_DTYPES[args.model_dtype]
    peaks = c.peaks
    sustained = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    c.clk.start()
    try:
        # ---- headline: the config batch-sharded over the ranks ----
        head, model, x = measure_sharded(c, cfg, args.steps, args.warmup, "headline", mdt, keep=True)
        ms_per_step = head["latency_ms"]
        tokens = cfg.batch_size * cfg.seq_len
        value = tokens / (ms_per_step / 1000.0)

        # ---- end to end through the public module: pinned host in, host out ----
        x_host = x.cpu().pin_memory()
        y_host = torch.empty_like(x_host).pin_memory()
        with torch.inference_mode():
            e2e_serial(model, x_host, y_host, 2, device, c.flush_buf)
            barrier(dist)
            with c.clk.window("e2e"):
                e_ts = e2e_serial(model, x_host, y_host, args.steps, device, c.flush_buf)
            barrier(dist)
            e_ms = max_over_ranks(sum(e_ts) / args.steps, dist, device)
            e2e_pipelined(model, x_host, y_host, 2, device)  # warm-up (streams)
            barrier(dist)
            with c.clk.window("e2e"):
                p_total = e2e_pipelined(model, x_host, y_host, args.steps, device)
            barrier(dist)
            p_ms = max_over_ranks(p_total / args.steps, dist, device)

        # ---- per-kernel roofline from an instrumented eager forward ----
        prof = kernel_profile(model, x)
        n_g, ms_g, fl_g = prof["gemm"]
        n_f, ms_f, fl_f = prof["flash"]
        n_l, ms_l, by_l = prof["ln"]
        gemm_tflops = fl_g / (ms_g / 1e3) / 1e12
        flash_tflops = fl_f / (ms_f / 1e3) / 1e12
        ln_gbs = by_l / (ms_l / 1e3) / 1e9
        launches_per_step = n_g + n_f + n_l
        rows = x.shape[0] * x.shape[1]
        del model, x
        torch.cuda.empty_cache()

        line = {
            "metric": f"forward tokens/s ({args.config})", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if mdt == torch.bfloat16 else "f16",
            "data": "synthetic",
            "config": {"workload": args.config, **cfg_dict(cfg), "global_batch": cfg.batch_size,
                       "rank_batch": head["rank_batch"], "parallelism": f"dp{world}",
                       "l2": "flushed between steps (256 MB write)", "weights": "default init, seed 0",
                       "cuda_graph": True, "model_dtype": args.model_dtype},
            "mfu": head["mfu"], "latency_ms": ms_per_step, "latency_ms_median": head["latency_ms_median"],
            "e2e": {"value": tokens / (e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
                    "d2h_bytes_per_step": y_host.numel() * y_host.element_size() * world,
                    "ms_per_step": e_ms,
                    "copies": "serial per step: pinned H2D of the step's input, forward, D2H of its output, "
                              "one event pair around the three",
                    "pipelined": {"value": tokens / (p_ms / 1e3), "ms_per_step": p_ms,
                                  "copies": "two copy streams; step i+1's upload and step i-1's download "
                                            "overlap step i's forward"}},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": {"bound": "tensor", "kernel": "gemm_f16_tcgen05", "achieved": gemm_tflops,
                         "peak": sustained, "unit": "TFLOP/s", "frac": gemm_tflops / sustained,
                         "peak_source": f"bf16_tflops_sustained ({c.peak_src}): the GEMMs are timed inside the step",
                         "frac_of_burst": gemm_tflops / peaks["bf16_tflops"],
                         "traffic": (C3_GEMM_DRAM_BYTES_PER_LAUNCH
                                     if args.config == "c3" and mdt == torch.float32 and world == 1 else None),
                         "traffic_unit": "bytes per launch (ncu dram read+write, c3 at one GPU)",
                         "algorithmic_bytes_per_launch": algo_bytes_per_gemm(cfg, 4 if mdt == torch.float32 else 2,
                                                                             rows),
                         "launches_per_step": n_g, "gemm_share_of_step": ms_g / ms_per_step},
            "kernels": {
                "flash_fwd_tcgen05": {"launches": n_f, "ms": ms_f, "tflops": flash_tflops,
                                      "frac": flash_tflops / sustained,
                                      "frac_of_burst": flash_tflops / peaks["bf16_tflops"]},
                "ln_residual": {"launches": n_l, "ms": ms_l, "gbs": ln_gbs, "frac": ln_gbs / peaks["hbm_gbs"]},
                "gemm_f16_tcgen05": {"launches": n_g, "ms": ms_g, "tflops": gemm_tflops},
            },
        }
        extra_steps = max(10, args.steps // 2)
        per = {}
        if not args.no_extra and args.config == "c3" and mdt == torch.float32:
            # ---- c5 context parallel and c4 batch-sharded at this N ----
            line["c5_cp"] = measure_cp(c, NAMED_CONFIGS["c5"], extra_steps, 2, "c5_cp")
            c4, _, _ = measure_sharded(c, NAMED_CONFIGS["c4"], extra_steps, 2, "c4_dp")
            line["c4_dp"] = c4
            if world > 1:
                weak = NAMED_CONFIGS["c3"]
                wk, _, _ = measure_sharded_weak(c, weak, extra_steps, "weak")
                line["weak"] = wk
            per["c3"] = {k: head[k] for k in ("latency_ms", "latency_ms_median", "tokens_per_s", "mfu")}
            per["c4"] = {k: c4[k] for k in ("latency_ms", "latency_ms_median", "tokens_per_s", "mfu")}
            per["c5"] = {k: line["c5_cp"][k] for k in ("latency_ms", "latency_ms_median", "tokens_per_s", "mfu")}
            if world == 1:
                for name in ("c1", "c2"):
                    r, _, _ = measure_sharded(c, NAMED_CONFIGS[name], max(20, args.steps), 3, name)
                    per[name] = {k: r[k] for k in ("latency_ms", "latency_ms_median", "tokens_per_s", "mfu")}
                    if name == "c2":
                        # weight-streaming floor: every fp16 weight read once at the measured HBM rate
                        cc = NAMED_CONFIGS[name]
                        wbytes = 2 * cc.num_layers * (4 * cc.d_model ** 2 + 2 * cc.d_model * cc.ffn_dim)
                        floor_ms = wbytes / (peaks["hbm_gbs"] * 1e9) * 1e3
                        per[name]["weight_floor_ms"] = floor_ms
                        per[name]["frac_of_weight_floor"] = floor_ms / r["latency_ms"]
            for name, v in per.items():
                v["bound"] = "launch/latency" if name in ("c1", "c2") else "tensor"
                v["parallelism"] = ("replica (N=1)" if name in ("c1", "c2")
                                    else (f"cp{world}" if name == "c5" else f"dp{world}"))
            line["per_config"] = dict(sorted(per.items()))
    finally:
        c.clk.stop()
    line["clocks"] = c.clk.summary()
    line["clocks_headline"] = c.clk.summary(["headline"])
    if world == 1 and not args.no_extra:
        threads = os.cpu_count() or 1
        times = cpu_reference_forward(cfg, threads, cfg.batch_size, 3)
        t = statistics.median(times)
        line["cpu_baseline"] = {"value": cfg.batch_size * cfg.seq_len / t, "unit": "tokens/s", "cores": threads,
                                "cpu_model": cpu_model(), "kind": "port", "latency_ms": t * 1e3,
                                "sample": f"full {args.config} forward ({cfg.batch_size} x {cfg.seq_len} tokens, "
                                          f"{cfg.num_layers} layers), median of {len(times)}",
                                "extrapolated": False}
    if rank == 0:
        emit(line)


def measure_sharded_weak(c: Ctx, cfg, steps, window):
    """Every rank runs the whole batch (weak scaling): value = all ranks'
    tokens / the slowest rank's time."""
    model = build_model(cfg, c.device)
    x = seeded_input(cfg, c.device, torch.float32, 0, cfg.batch_size)
    with torch.inference_mode():
        for _ in range(3):
            model(x)
    barrier(c.dist)
    with c.clk.window(window):
        with torch.inference_mode():
            ts = time_steps(lambda: model(x), steps, c.flush_buf)
    barrier(c.dist)
    ms = max_over_ranks(sum(ts) / steps, c.dist, c.device)
    tokens = c.world * cfg.batch_size * cfg.seq_len
    del model, x
    torch.cuda.empty_cache()
    return {"latency_ms": ms, "tokens_per_s": tokens / (ms / 1e3), "global_batch": c.world * cfg.batch_size,
            "scaling": "weak", "steps": steps}, None, None


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[1])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3", choices=sorted(NAMED_CONFIGS))
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-extra", action="store_true",
                    help="headline only: skip c5_cp, c4_dp, weak, per_config and cpu_baseline")
    ap.add_argument("--model-dtype", default="float32", choices=sorted(MODEL_DTYPES),
                    help="parameter and input dtype of the model (the BASELINE configs are float32)")
    args = ap.parse_args()
    # stdout carries exactly the JSON line: the libraries' own prints (NCCL's
    # version banner, for one) are sent to stderr at the file-descriptor level
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
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
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        # high-priority NCCL streams: the ring's send/recv kernels then take
        # the next free SMs ahead of the flash kernel's waiting CTAs
        opts = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank), pg_options=opts)
    try:
        if world > 1 and cfg.batch_size < world:
            if args.model_dtype != "float32":
                raise SystemExit("context parallelism runs the float32 model")
            run_cp_headline(args, cfg, rank, world, local_rank)
        else:
            run_ours(args, cfg, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


def run_cp_headline(args, cfg, rank, world, local_rank):
    """--config c5 (one sequence) at N > 1: the context-parallel forward is
    the headline."""
    import torch.distributed as dist
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    c = Ctx(args, rank, world, local_rank, dist)
    c.clk.start()
    try:
        r = measure_cp(c, cfg, args.steps, args.warmup, "headline")
    finally:
        c.clk.stop()
    tokens = cfg.batch_size * cfg.seq_len
    line = {
        "metric": f"forward tokens/s ({args.config})", "value": r["tokens_per_s"], "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["latency_ms"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": args.config, **cfg_dict(cfg), "global_batch": cfg.batch_size,
                   "parallelism": r["parallelism"], "layout": r["layout"], "shard_tokens": r["shard_tokens"],
                   "l2": "flushed between steps (256 MB write)", "weights": "default init, seed 0",
                   "cuda_graph": False},
        "mfu": r["mfu"], "latency_ms": r["latency_ms"], "e2e": r["e2e"],
        "gpu_launches": (cfg.num_layers * (6 + 2 * world) + 1) * args.steps,
        "ring": r.get("ring"), "clocks": c.clk.summary(), "tokens": tokens,
    }
    if rank == 0:
        emit(line)


if __name__ == "__main__":
    raise SystemExit(main())
