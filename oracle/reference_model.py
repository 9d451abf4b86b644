"""TEST INFRASTRUCTURE ONLY - the parity oracle, never the product.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may
import this module, and only to check or to time the reference algorithm on the
host. The product path (`transformer_optimization_b200`) never imports it.

A plain fp32 PyTorch restatement of the reference's eager model
`BaselineTransformer` (torch_transformer_benchmark.py:135-248) and of its
memory-bounded twin `QueryTiledBaselineTransformer`
(torch_transformer_benchmark.py:341-437), written as functions over a
`state_dict` so that it needs no module classes from either side. Every step
keeps the reference's operation order (scale AFTER QK^T, masked_fill with
-inf, softmax in fp32, exact-erf GELU, pre-LN residual blocks, final LN and the
trailing padding masks).

Pinning: `tests/golden/make_golden.py` imports the real reference in the build
container and records its outputs; `tests/test_oracle_golden.py` checks this
file against them (bit-for-bit equal on CPU for the same torch build, and to
1e-5 otherwise).

Also here: the accuracy gate `compare_outputs` (torch_transformer_benchmark.py:
4548-4615, the exact OR criterion, not isclose) and the seeded input protocol.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

Params = Dict[str, torch.Tensor]


# --------------------------------------------------------------------------
# Model pieces (torch_transformer_benchmark.py:135-248)
# --------------------------------------------------------------------------

def _linear(p: Params, name: str, x: torch.Tensor) -> torch.Tensor:
    return F.linear(x, p[name + ".weight"], p[name + ".bias"])


def _layer_norm(p: Params, name: str, x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    w = p[name + ".weight"]
    return F.layer_norm(x, (w.shape[0],), w, p[name + ".bias"], eps)


def _split_heads(x: torch.Tensor, heads: int) -> torch.Tensor:
    """[B,S,D] -> [B,H,S,hd] (torch_transformer_benchmark.py:154-160)."""
    b, s, d = x.shape
    return x.view(b, s, heads, d // heads).transpose(1, 2).contiguous()


def attention(p: Params, prefix: str, x: torch.Tensor, heads: int,
              valid_token_mask: Optional[torch.Tensor], causal: bool) -> torch.Tensor:
    """BaselineSelfAttention.forward (torch_transformer_benchmark.py:162-200)."""
    b, s, d = x.shape
    hd = d // heads
    scale = hd ** -0.5
    q = _split_heads(_linear(p, prefix + ".q_proj", x), heads)
    k = _split_heads(_linear(p, prefix + ".k_proj", x), heads)
    v = _split_heads(_linear(p, prefix + ".v_proj", x), heads)
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        cm = torch.ones((s, s), device=x.device, dtype=torch.bool).triu(diagonal=1)
        scores = scores.masked_fill(cm, float("-inf"))
    if valid_token_mask is not None:
        scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)
    ctx = torch.matmul(probs, v).transpose(1, 2).contiguous().view(b, s, d)
    out = _linear(p, prefix + ".out_proj", ctx)
    if valid_token_mask is not None:
        out = out.masked_fill(~valid_token_mask[..., None], 0)
    return out


def attention_query_tiled(p: Params, prefix: str, x: torch.Tensor, heads: int,
                          valid_token_mask: Optional[torch.Tensor], causal: bool,
                          query_tile: int) -> torch.Tensor:
    """QueryTiledBaselineSelfAttention.forward (torch_transformer_benchmark.py:
    353-421): full K/V, query rows in tiles, fp32 softmax per tile. Exactly the
    dense attention, with a bounded score buffer."""
    b, s, d = x.shape
    hd = d // heads
    scale = hd ** -0.5
    q = _split_heads(_linear(p, prefix + ".q_proj", x), heads)
    k = _split_heads(_linear(p, prefix + ".k_proj", x), heads)
    v = _split_heads(_linear(p, prefix + ".v_proj", x), heads)
    ctx = torch.empty_like(q)
    kt = k.transpose(-2, -1)
    for start in range(0, s, query_tile):
        end = min(start + query_tile, s)
        scores = torch.matmul(q[:, :, start:end], kt) * scale
        if causal:
            qp = torch.arange(start, end, device=x.device)[:, None]
            kp = torch.arange(s, device=x.device)[None, :]
            scores.masked_fill_(kp > qp, float("-inf"))
        if valid_token_mask is not None:
            scores.masked_fill_(~valid_token_mask[:, None, None, :], float("-inf"))
        ctx[:, :, start:end] = torch.matmul(torch.softmax(scores.float(), dim=-1).to(x.dtype), v)
    ctx = ctx.transpose(1, 2).contiguous().view(b, s, d)
    out = _linear(p, prefix + ".out_proj", ctx)
    if valid_token_mask is not None:
        out = out.masked_fill(~valid_token_mask[..., None], 0)
    return out


def ffn(p: Params, prefix: str, x: torch.Tensor, row_chunk: Optional[int] = None) -> torch.Tensor:
    """ffn_out(gelu_erf(ffn_in(x))) (torch_transformer_benchmark.py:224), with
    the optional row chunking of ChunkedBaselineTransformerBlock
    (torch_transformer_benchmark.py:296-305)."""
    if row_chunk is None:
        return _linear(p, prefix + ".ffn_out",
                       F.gelu(_linear(p, prefix + ".ffn_in", x), approximate="none"))
    b, s, d = x.shape
    flat = x.reshape(b * s, d)
    out = torch.empty_like(flat)
    for start in range(0, flat.shape[0], row_chunk):
        piece = flat[start:start + row_chunk]
        out[start:start + row_chunk] = _linear(
            p, prefix + ".ffn_out", F.gelu(_linear(p, prefix + ".ffn_in", piece), approximate="none"))
    return out.view(b, s, d)


def forward(p: Params, cfg, x: torch.Tensor,
            valid_token_mask: Optional[torch.Tensor] = None,
            query_tile: Optional[int] = None,
            ffn_row_chunk: Optional[int] = None,
            layers: Optional[int] = None) -> torch.Tensor:
    """BaselineTransformer.forward (torch_transformer_benchmark.py:238-248) with
    BaselineTransformerBlock.forward (torch_transformer_benchmark.py:215-228).

    `query_tile` switches the attention to the query-tiled reference
    (QueryTiledBaselineTransformer, torch_transformer_benchmark.py:424-437),
    `ffn_row_chunk` to the row-chunked FFN. `layers` limits the stack to its
    first layers (used only to time a bounded slice of a large config)."""
    n_layers = cfg.num_layers if layers is None else layers
    for i in range(n_layers):
        pre = f"layers.{i}"
        h = _layer_norm(p, pre + ".norm1", x)
        if query_tile is None:
            a = attention(p, pre + ".attention", h, cfg.num_heads, valid_token_mask, cfg.causal)
        else:
            a = attention_query_tiled(p, pre + ".attention", h, cfg.num_heads,
                                      valid_token_mask, cfg.causal, query_tile)
        x = x + a
        x = x + ffn(p, pre, _layer_norm(p, pre + ".norm2", x), ffn_row_chunk)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
    x = _layer_norm(p, "final_norm", x)
    if valid_token_mask is not None:
        x = x.masked_fill(~valid_token_mask[..., None], 0)
    return x


# --------------------------------------------------------------------------
# Parameters, seeded inputs (BASELINE protocol) and the reference harness's
# random case generator (torch_transformer_benchmark.py:4359-4397)
# --------------------------------------------------------------------------

def init_params(cfg, seed: Optional[int] = 0) -> Params:
    """Default-initialised parameters in the exact construction order of
    BaselineTransformer.__init__ (torch_transformer_benchmark.py:230-236,
    203-209, 142-152): per layer norm1, q/k/v/out_proj, norm2, ffn_in,
    ffn_out; then final_norm. nn.Linear draws kaiming_uniform(a=sqrt(5)) for
    the weight (= U(+-1/sqrt(fan_in))) then U(+-1/sqrt(fan_in)) for the bias;
    LayerNorm is weight=1, bias=0 and draws nothing. With `seed` the global
    RNG is reseeded first, as `torch.manual_seed(0); BaselineTransformer(cfg)`
    does."""
    if seed is not None:
        torch.manual_seed(seed)
    d, f = cfg.d_model, cfg.ffn_dim
    p: Params = {}

    def linear(name: str, out_f: int, in_f: int) -> None:
        w = torch.empty(out_f, in_f)
        torch.nn.init.kaiming_uniform_(w, a=math.sqrt(5))
        bound = 1.0 / math.sqrt(in_f)
        b = torch.empty(out_f).uniform_(-bound, bound)
        p[name + ".weight"] = w
        p[name + ".bias"] = b

    def norm(name: str, n: int) -> None:
        p[name + ".weight"] = torch.ones(n)
        p[name + ".bias"] = torch.zeros(n)

    for i in range(cfg.num_layers):
        pre = f"layers.{i}"
        norm(pre + ".norm1", d)
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            linear(f"{pre}.attention.{proj}", d, d)
        norm(pre + ".norm2", d)
        linear(pre + ".ffn_in", f, d)
        linear(pre + ".ffn_out", d, f)
    norm("final_norm", d)
    return p


def seeded_case(cfg, seed: int = 0) -> Tuple[Params, torch.Tensor]:
    """The benchmark definition's protocol: torch.manual_seed(seed), build the
    model (default init), then x = torch.randn(B, S, D) on the CPU."""
    p = init_params(cfg, seed)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model)
    return p, x


def padded_mask(cfg, padding_ratio: float, seed: int) -> torch.Tensor:
    """Key-padding mask with per-row valid lengths drawn like
    generate_random_case (torch_transformer_benchmark.py:4386-4396), but from a
    CPU generator so it is the same on every machine."""
    g = torch.Generator()
    g.manual_seed(seed)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(min_valid, cfg.seq_len + 1, (cfg.batch_size,), generator=g)
    return torch.arange(cfg.seq_len)[None, :] < lengths[:, None]


def harness_case(cfg, device, dtype: torch.dtype, seed: int, padding_ratio: float,
                 input_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """generate_random_case (torch_transformer_benchmark.py:4359-4397), the
    harness's per-trial input: x ~ N(0,1) * input_scale from a generator on
    `device` seeded with `seed`; with padding_ratio > 0, per-row valid lengths
    drawn from the same generator and x zeroed at the padded tokens; the mask
    is all True otherwise (the harness always passes one)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, generator=g, device=device, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(cfg.batch_size, cfg.seq_len, device=device, dtype=torch.bool)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=cfg.seq_len + 1, size=(cfg.batch_size,), generator=g,
                            device=device)
    mask = torch.arange(cfg.seq_len, device=device)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


# --------------------------------------------------------------------------
# Accuracy gate (torch_transformer_benchmark.py:4534-4615)
# --------------------------------------------------------------------------

@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float
    failed_feature_dims: List[int]


def compare_outputs(reference: torch.Tensor, optimized: torch.Tensor,
                    rtol: float = 0.02, atol: float = 0.002) -> AccuracyResult:
    """finite & (|opt-ref| <= atol | |opt-ref| <= rtol*|ref|), zero failures
    to pass - the exact OR criterion of torch_transformer_benchmark.py:
    4571-4575 (deliberately not torch.isclose's atol + rtol*|ref|)."""
    if reference.shape != optimized.shape:
        raise AssertionError(f"shape mismatch: baseline={tuple(reference.shape)}, "
                             f"optimized={tuple(optimized.shape)}")
    ref = reference.detach().float()
    opt = optimized.detach().float().to(ref.device)
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    err = (opt - ref).abs()
    ok = finite & ((err <= atol) | (err <= rtol * ref.abs()))
    failed = ~ok
    n_failed = int(failed.sum().item())
    flat = int(err.reshape(-1).argmax().item())
    idx = []
    for size in reversed(reference.shape):
        idx.append(flat % size)
        flat //= size
    worst = tuple(reversed(idx))
    rel = err / ref.abs().clamp_min(1e-12)
    if reference.ndim >= 2:
        dims = torch.nonzero(failed.any(dim=tuple(range(reference.ndim - 1))),
                             as_tuple=False).flatten().tolist()
    else:
        dims = torch.nonzero(failed, as_tuple=False).flatten().tolist()
    return AccuracyResult(
        passed=n_failed == 0,
        total_elements=reference.numel(),
        failed_elements=n_failed,
        max_abs_error=float(err.max().item()) if err.numel() else 0.0,
        max_relative_error=float(rel.max().item()) if rel.numel() else 0.0,
        mean_abs_error=float(err.mean().item()) if err.numel() else 0.0,
        worst_index=worst,
        reference_at_worst=float(ref[worst].item()) if ref.numel() else 0.0,
        optimized_at_worst=float(opt[worst].item()) if opt.numel() else 0.0,
        failed_feature_dims=dims,
    )


# --------------------------------------------------------------------------
# Per-op references used by the kernel parity tests. Each states the
# reference's fp16-GEMM-path arithmetic for one op
# (torch_transformer_benchmark.py:4130-4199).
# --------------------------------------------------------------------------

def ln_site(x: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor, b: torch.Tensor,
            eps: float, valid: Optional[torch.Tensor], mask_delta: bool, mask_x: bool,
            mask_out: bool) -> Tuple[torch.Tensor, torch.Tensor]:
    """_ln_site's ATen branch (torch_transformer_benchmark.py:3988-4001):
    delta -> fp32 -> zero invalid rows (mask_delta); x + delta; zero invalid
    rows (mask_x); LayerNorm; zero invalid rows (mask_out). Returns fp32
    (x_new, normed)."""
    x = x.float()
    inv = None if valid is None else (~valid.reshape(-1, 1).bool())
    if delta is not None:
        d = delta.float()
        if mask_delta:
            d = d.masked_fill(inv, 0)
        x = x + d
    if mask_x:
        x = x.masked_fill(inv, 0)
    y = F.layer_norm(x, (x.shape[-1],), w.float(), b.float(), eps)
    if mask_out:
        y = y.masked_fill(inv, 0)
    return x, y


def linear_fp16(a16: torch.Tensor, w16: torch.Tensor, b: torch.Tensor,
                gelu: bool) -> torch.Tensor:
    """fp16 operands, exact (fp64) accumulation, + bias, [exact-erf GELU],
    rounded once to fp16 - the projection of the reference's fp16-GEMM path
    (torch_transformer_benchmark.py:4138-4194, kernel 1756-1803) without its
    intermediate fp16 rounding of the bias and of the GELU input. Returns the
    fp16 result as fp32 values."""
    h = a16.double() @ w16.double().t() + b.double()
    if gelu:
        h = F.gelu(h, approximate="none")
    return h.float().half().float()


def linear_residual(a16: torch.Tensor, w: torch.Tensor, b: torch.Tensor, x_in: torch.Tensor,
                    valid: Optional[torch.Tensor], mask_delta: bool, mask_x: bool) -> torch.Tensor:
    """x_in + mask_delta(a16 @ w^T + b), then mask_x, in fp64 rounded to fp32:
    the residual add of the reference's LayerNorm sites
    (torch_transformer_benchmark.py:3988-3995) applied to a projection output
    kept in full precision. `w` is the weight the product should see (fp16
    values, or the fp32 weight for split-weight GEMMs)."""
    delta = a16.double() @ w.double().t() + b.double()
    if valid is not None and mask_delta:
        delta = delta.masked_fill(~valid.reshape(-1, 1).bool(), 0)
    y = x_in.double() + delta
    if valid is not None and mask_x:
        y = y.masked_fill(~valid.reshape(-1, 1).bool(), 0)
    return y.float()


# Half-precision models (parameters and activations in T = fp16 or bf16): the
# eager model run in T stores every op's output in T
# (torch_transformer_benchmark.py:162-248 with T tensors). These restate the
# roundings of one kernel call of that path, from exact (fp64) products.

def ln_site_half(x: torch.Tensor, delta: Optional[torch.Tensor], w: torch.Tensor, b: torch.Tensor,
                 eps: float, valid: Optional[torch.Tensor], mask_delta: bool, mask_x: bool,
                 mask_out: bool, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """`x = x + delta` stored in T (torch_transformer_benchmark.py:218-222),
    then nn.LayerNorm of the T tensor (fp32 statistics, output rounded to T by
    the caller's comparison), with the masking points of ln_site. x, delta in
    T; returns fp32 (x_new with T values, normed before its rounding)."""
    xf = x.float()
    inv = None if valid is None else (~valid.reshape(-1, 1).bool())
    if delta is not None:
        d = delta.float()
        if mask_delta:
            d = d.masked_fill(inv, 0)
        xf = (xf + d).to(dtype).float()
    if mask_x:
        xf = xf.masked_fill(inv, 0)
    y = F.layer_norm(xf, (xf.shape[-1],), w.float(), b.float(), eps)
    if mask_out:
        y = y.masked_fill(inv, 0)
    return xf, y


def linear_half(a: torch.Tensor, w: torch.Tensor, b: torch.Tensor, gelu: bool,
                dtype: torch.dtype) -> torch.Tensor:
    """T(a @ w^T + b) from an exact (fp64) product, and with `gelu` the exact-
    erf GELU of that stored T value, rounded to T again: nn.Linear then F.gelu
    on T tensors (torch_transformer_benchmark.py:224). Returns fp32 values."""
    h = (a.double() @ w.double().t() + b.double()).to(dtype)
    if gelu:
        h = F.gelu(h.double(), approximate="none").to(dtype)
    return h.float()


def linear_residual_half(a: torch.Tensor, w: torch.Tensor, b: torch.Tensor, x_in: torch.Tensor,
                         valid: Optional[torch.Tensor], mask_delta: bool, mask_x: bool,
                         dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """x = T(x + T(a @ w^T + b)) with the masking points of linear_residual:
    the out_proj / ffn_out output stored in T, then the residual add stored in
    T (torch_transformer_benchmark.py:197-200, 218-226). Returns fp32
    (x_new, the stored projection)."""
    v = (a.double() @ w.double().t() + b.double()).to(dtype).double()
    if valid is not None and mask_delta:
        v = v.masked_fill(~valid.reshape(-1, 1).bool(), 0)
    y = (x_in.double() + v).to(dtype).double()
    if valid is not None and mask_x:
        y = y.masked_fill(~valid.reshape(-1, 1).bool(), 0)
    return y.float(), v.float()


def attention_fp16(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                   causal: bool, key_valid: Optional[torch.Tensor] = None,
                   q_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """softmax(scale * Q K^T) V in fp32 from fp16-valued q/k/v [B,H,S,hd];
    causal masks key j > query i + q_offset. Returns (out [B,H,Sq,hd] fp32,
    lse [B,H,Sq] natural-log sum-exp of the scaled scores). Rows whose keys
    are all masked give out=0, lse=-inf."""
    s = torch.matmul(q.float(), k.float().transpose(-2, -1)) * scale
    sq, sk = q.shape[-2], k.shape[-2]
    if causal:
        qi = torch.arange(sq)[:, None] + q_offset
        kj = torch.arange(sk)[None, :]
        s = s.masked_fill((kj > qi).to(s.device), float("-inf"))
    if key_valid is not None:
        s = s.masked_fill(~key_valid[:, None, None, :].to(s.device), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    return torch.matmul(p, v.float()), lse


def attention_rounded_scores(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                             causal: bool, key_valid: Optional[torch.Tensor] = None,
                             q_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """attention_fp16 on T-valued q/k/v [B,H,S,hd] (T = q.dtype, fp16 or
    bf16) with the scores the eager model computes in T:
    T(T(q k^T) * scale) - the product accumulated in fp32 and rounded once
    to T, then the scale applied in fp32 and rounded to T
    (torch_transformer_benchmark.py:173) - then the fp32 softmax (:188) and
    an fp32 P V. Returns (out fp32, lse of the rounded scores)."""
    dt = q.dtype
    s = torch.matmul(q.float(), k.float().transpose(-2, -1)).to(dt)
    s = (s.float() * float(scale)).to(dt).float()
    sq, sk = q.shape[-2], k.shape[-2]
    if causal:
        qi = torch.arange(sq)[:, None] + q_offset
        kj = torch.arange(sk)[None, :]
        s = s.masked_fill((kj > qi).to(s.device), float("-inf"))
    if key_valid is not None:
        s = s.masked_fill(~key_valid[:, None, None, :].to(s.device), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.nan_to_num(torch.exp(s - lse[..., None]), nan=0.0)
    return torch.matmul(p, v.float()), lse
