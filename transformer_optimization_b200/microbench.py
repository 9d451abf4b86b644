"""Kernel micro-benchmark: time one kernel in isolation with CUDA events.

    python -m transformer_optimization_b200.microbench gemm  M N K [--gelu] [--tile-n T]
    python -m transformer_optimization_b200.microbench flash B H S HD [--causal]
    python -m transformer_optimization_b200.microbench ln    M D
    python -m transformer_optimization_b200.microbench merge B S H HD

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


def _time(fn, warmup, iters, min_warm_s=0.3, min_time_s=0.2):
    """Mean ms per launch. Warm-up runs at least `warmup` launches and
    `min_warm_s` seconds (so clocks have ramped); the timed loop runs at
    least `iters` launches and `min_time_s` seconds."""
    import time
    t0 = time.perf_counter()
    n = 0
    while n < warmup or (min_warm_s > 0 and time.perf_counter() - t0 < min_warm_s):
        fn()
        n += 1
        if n % 16 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    # size the timed loop from one measured launch
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    fn()
    e.record()
    torch.cuda.synchronize()
    one = max(s.elapsed_time(e), 1e-3)
    reps = max(iters, int(min_time_s * 1e3 / one))
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=("gemm", "gemm_res", "flash", "ln", "merge"))
    ap.add_argument("dims", type=int, nargs="+")
    ap.add_argument("--gelu", action="store_true")
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--pure", action="store_true", help="ln: LayerNorm only (no residual delta, no x write)")
    ap.add_argument("--exp-f16x2", action="store_true", help="flash: packed fp16 exp2 path")
    ap.add_argument("--fma-exp", type=int, default=0, help="flash: pairs per row exponentiated on the FMA pipes")
    ap.add_argument("--tile-n", type=int, default=0)
    ap.add_argument("--pair", type=int, default=0, help="0 auto, 1 one-CTA tiles, 2 two-SM tiles")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--min-warm-s", type=float, default=0.3, help="minimum warm-up seconds (0 for ncu)")
    ap.add_argument("--min-time-s", type=float, default=0.2, help="minimum timed seconds (0 for ncu)")
    a = ap.parse_args(argv)
    T = lambda fn: _time(fn, a.warmup, a.iters, a.min_warm_s, a.min_time_s)
    torch.manual_seed(0)
    dev = torch.device("cuda")
    if a.kernel == "gemm":
        m, n, k = a.dims
        x = torch.randn(m, k, device=dev).half()
        w = (torch.randn(n, k, device=dev) / math.sqrt(k)).half()
        b = torch.randn(n, device=dev)
        out = torch.empty(m, n, device=dev, dtype=torch.float16)
        ms = T(lambda: K.linear(x, w, b, gelu=a.gelu, out=out, tile_n=a.tile_n, pair=a.pair))
        rate = 2.0 * m * n * k / (ms / 1e3) / 1e12
        print(f"gemm M={m} N={n} K={k} gelu={a.gelu} tile_n={a.tile_n} pair={a.pair}: {ms:.4f} ms  "
              f"{rate:.1f} TFLOP/s")
    elif a.kernel == "gemm_res":
        m, n, k = a.dims
        x = torch.randn(m, k, device=dev).half()
        w = (torch.randn(n, k, device=dev) / math.sqrt(k)).half()
        b = torch.randn(n, device=dev)
        xr = torch.randn(m, n, device=dev)
        ms = T(lambda: K.linear_residual(x, w, b, xr, xr, tile_n=a.tile_n, pair=a.pair))
        rate = 2.0 * m * n * k / (ms / 1e3) / 1e12
        print(f"gemm_res M={m} N={n} K={k} tile_n={a.tile_n} pair={a.pair}: {ms:.4f} ms  {rate:.1f} TFLOP/s")
    elif a.kernel == "flash":
        bsz, h, s, hd = a.dims
        d = h * hd
        qkv = torch.randn(bsz, s, 3 * d, device=dev).half()
        out = torch.empty(bsz, s, d, device=dev, dtype=torch.float16)
        ms = T(lambda: K.flash_attention(qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:], h, hd ** -0.5,
                                         causal=a.causal, out=out, exp_f16x2=a.exp_f16x2,
                                         fma_exp_pairs=a.fma_exp))
        flops = 4.0 * bsz * s * s * d * (0.5 if a.causal else 1.0)
        print(f"flash B={bsz} H={h} S={s} hd={hd} causal={a.causal}: {ms:.4f} ms  "
              f"{flops / (ms / 1e3) / 1e12:.1f} TFLOP/s")
    elif a.kernel == "merge":
        # one ring step's combine (context parallelism): fp32 accumulator and
        # partial [B, S, H*hd] with their [B, H, S] log-sum-exps, fp16 copy out
        bsz, s, h, hd = a.dims
        d = h * hd
        o_acc = torch.randn(bsz, s, d, device=dev)
        o_part = torch.randn(bsz, s, d, device=dev)
        lse_acc = torch.randn(bsz, h, s, device=dev)
        lse_part = torch.randn(bsz, h, s, device=dev)
        out16 = torch.empty(bsz, s, d, device=dev, dtype=torch.float16)
        ms = T(lambda: K.attn_merge(o_acc, lse_acc, o_part, lse_part, h, out16=out16))
        nbytes = bsz * s * d * (4 + 4 + 4 + 2) + bsz * h * s * 4 * 3  # o_acc r+w, o_part r, fp16 out; lse r, r, w
        print(f"merge B={bsz} S={s} H={h} hd={hd}: {ms:.4f} ms  {nbytes / (ms / 1e3) / 1e9:.1f} GB/s")
    else:
        m, d = a.dims
        x = torch.randn(m, d, device=dev)
        delta = torch.randn(m, d, device=dev).half()
        w = torch.ones(d, device=dev)
        b = torch.zeros(d, device=dev)
        xo = torch.empty_like(x)
        nrm = torch.empty(m, d, device=dev, dtype=torch.float16)
        if a.pure:  # the model's LayerNorm sites: read x, write fp16 normed
            ms = T(lambda: K.ln_residual(x, None, w, b, 1e-5, normed=nrm))
            print(f"ln (pure) M={m} D={d}: {ms:.4f} ms  {m * d * 6 / (ms / 1e3) / 1e9:.1f} GB/s")
        else:
            ms = T(lambda: K.ln_residual(x, delta, w, b, 1e-5, write_x=True, x_out=xo, normed=nrm))
            print(f"ln M={m} D={d}: {ms:.4f} ms  {m * d * 12 / (ms / 1e3) / 1e9:.1f} GB/s")


if __name__ == "__main__":
    main()
