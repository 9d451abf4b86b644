"""Kernel micro-benchmark: time one kernel in isolation with CUDA events.

    python -m transformer_optimization_b200.microbench gemm  M N K [--gelu] [--tile-n T]
    python -m transformer_optimization_b200.microbench flash B H S HD [--causal]
    python -m transformer_optimization_b200.microbench ln    M D

Prints one line: kernel, shape, mean time per launch (ms) and the achieved
rate against its roofline unit (TFLOP/s for GEMM/attention, GB/s for
LayerNorm). Inputs are seeded random; --iters launches are timed after
--warmup untimed ones. Also the command used for the committed ncu captures
(small cases, single kernel).
"""

from __future__ import annotations

import argparse
import math

import torch

from . import kernels as K


def _time(fn, warmup, iters):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=("gemm", "flash", "ln"))
    ap.add_argument("dims", type=int, nargs="+")
    ap.add_argument("--gelu", action="store_true")
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--tile-n", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    torch.manual_seed(0)
    dev = torch.device("cuda")
    if a.kernel == "gemm":
        m, n, k = a.dims
        x = torch.randn(m, k, device=dev).half()
        w = (torch.randn(n, k, device=dev) / math.sqrt(k)).half()
        b = torch.randn(n, device=dev).half()
        out = torch.empty(m, n, device=dev, dtype=torch.float16)
        ms = _time(lambda: K.linear(x, w, b, gelu=a.gelu, out=out, tile_n=a.tile_n), a.warmup, a.iters)
        rate = 2.0 * m * n * k / (ms / 1e3) / 1e12
        print(f"gemm M={m} N={n} K={k} gelu={a.gelu} tile_n={a.tile_n}: {ms:.4f} ms  {rate:.1f} TFLOP/s")
    elif a.kernel == "flash":
        bsz, h, s, hd = a.dims
        d = h * hd
        qkv = torch.randn(bsz, s, 3 * d, device=dev).half()
        out = torch.empty(bsz, s, d, device=dev, dtype=torch.float16)
        ms = _time(lambda: K.flash_attention(qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:], h, hd ** -0.5,
                                             causal=a.causal, out=out), a.warmup, a.iters)
        flops = 4.0 * bsz * s * s * d * (0.5 if a.causal else 1.0)
        print(f"flash B={bsz} H={h} S={s} hd={hd} causal={a.causal}: {ms:.4f} ms  "
              f"{flops / (ms / 1e3) / 1e12:.1f} TFLOP/s")
    else:
        m, d = a.dims
        x = torch.randn(m, d, device=dev)
        delta = torch.randn(m, d, device=dev).half()
        w = torch.ones(d, device=dev)
        b = torch.zeros(d, device=dev)
        xo = torch.empty_like(x)
        nrm = torch.empty(m, d, device=dev, dtype=torch.float16)
        ms = _time(lambda: K.ln_residual(x, delta, w, b, 1e-5, write_x=True, x_out=xo, normed=nrm),
                   a.warmup, a.iters)
        print(f"ln M={m} D={d}: {ms:.4f} ms  {m * d * 12 / (ms / 1e3) / 1e9:.1f} GB/s")


if __name__ == "__main__":
    main()
