"""The drop-in module: `UserOptimizedTransformer` on B200 kernels.

Module tree, parameter names, shapes and construction order are those of the
reference's `BaselineTransformer` (torch_transformer_benchmark.py:135-248), so
`load_state_dict(strict=True)` accepts a reference state_dict and the default
initialisation under a given seed draws the same weights.

`UserOptimizedTransformer.forward(x, valid_token_mask=None)` keeps the
reference's contract (torch_transformer_benchmark.py:3509-3611): [B,S,D] in,
[B,S,D] out of x's dtype, the input is never mutated, the result never
aliases internal buffers, and nothing new is registered as a parameter or
buffer. For the fp32 model its arithmetic is the reference's fp32-model fast
path (torch_transformer_benchmark.py:4130-4199): every GEMM and the attention
run in fp16 with fp32 accumulation, residual stream and LayerNorm stay fp32.
fp16 and bf16 models (parameters and input of that type, T) run the same
kernels on T operands and keep the eager model's roundings to T: every
Linear output, the residual stream and the LayerNorm outputs are stored in T
(torch_transformer_benchmark.py:162-248 run in T). The kernels are this
package's sm_100a CUDA code reached through the C ABI; there is no eager/CPU
fallback.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn

from . import kernels
from .config import TransformerConfig


class BaselineSelfAttention(nn.Module):
    """Parameter container with the reference's layout
    (torch_transformer_benchmark.py:135-152): q/k/v/out_proj Linear(D, D)."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)

    def forward(self, *args, **kwargs):  # pragma: no cover - structure only
        raise NotImplementedError("run the whole model through UserOptimizedTransformer")


class BaselineTransformerBlock(nn.Module):
    """Parameter container with the reference's layout
    (torch_transformer_benchmark.py:202-209): norm1, attention, norm2,
    ffn_in Linear(D, F), ffn_out Linear(F, D)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = BaselineSelfAttention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, *args, **kwargs):  # pragma: no cover - structure only
        raise NotImplementedError("run the whole model through UserOptimizedTransformer")


class BaselineTransformer(nn.Module):
    """The reference model's module tree (torch_transformer_benchmark.py:
    230-236): `layers` of BaselineTransformerBlock, then `final_norm`.

    Here it is the parameter layout only. The eager fp32 reference forward is
    not part of this package (its restatement lives in the test oracle);
    calling it raises."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        config.validate()
        self.config = config
        self.layers = nn.ModuleList(
            [BaselineTransformerBlock(config.d_model, config.num_heads, config.ffn_dim)
             for _ in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        raise NotImplementedError(
            "BaselineTransformer here is the parameter layout only; use UserOptimizedTransformer "
            "(B200 kernels) or the reference's eager BaselineTransformer")


def copy_model_weights(baseline: nn.Module, optimized: nn.Module, strict: bool = True) -> None:
    """Copy identical weights into both implementations
    (torch_transformer_benchmark.py:4328-4338)."""
    incompatible = optimized.load_state_dict(
        {k: v.detach().clone() for k, v in baseline.state_dict().items()}, strict=strict)
    if not strict:
        if incompatible.missing_keys:
            print(f"[warning] missing optimized keys: {incompatible.missing_keys}")
        if incompatible.unexpected_keys:
            print(f"[warning] unexpected optimized keys: {incompatible.unexpected_keys}")


class _LayerWeights:
    """GEMM operands of one layer in the compute type `ct` (fp16 for the fp32
    and fp16 models, bf16 for bf16 models): packed [3D, D] QKV as the
    reference packs it (torch_transformer_benchmark.py:440-504), and fp32
    biases and LayerNorm parameters (exact for every model type). With
    `split_ffn_out` (fp32 model) the FFN-out weight is kept as [W_hi | W_lo]
    (kernels.split_weight) for a near-fp32 product."""

    __slots__ = ("wqkv", "bqkv", "wo", "bo", "w1", "b1", "w2", "b2", "split_w2", "n1w", "n1b", "n2w", "n2b")

    def __init__(self, blk: BaselineTransformerBlock, split_ffn_out: bool, ct: torch.dtype = torch.float16) -> None:
        at = blk.attention
        with torch.no_grad():
            self.wqkv = torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight], 0).to(ct).contiguous()
            self.bqkv = torch.cat([at.q_proj.bias, at.k_proj.bias, at.v_proj.bias], 0).float().contiguous()
            self.wo = at.out_proj.weight.to(ct).contiguous()
            self.bo = at.out_proj.bias.float().contiguous()
            self.w1 = blk.ffn_in.weight.to(ct).contiguous()
            self.b1 = blk.ffn_in.bias.float().contiguous()
            self.split_w2 = split_ffn_out
            self.w2 = (kernels.split_weight(blk.ffn_out.weight) if split_ffn_out
                       else blk.ffn_out.weight.to(ct).contiguous())
            self.b2 = blk.ffn_out.bias.float().contiguous()
            self.n1w = blk.norm1.weight.float().contiguous()
            self.n1b = blk.norm1.bias.float().contiguous()
            self.n2w = blk.norm2.weight.float().contiguous()
            self.n2b = blk.norm2.bias.float().contiguous()


def _splitk(m: int, n: int, k: int, sms: int) -> Optional[int]:
    """0 (automatic split count) when a projection of m rows should use the
    split-K form, else None: fewer than a quarter of the SMs would get a
    128 x 64 tile and K has at least 4 blocks of 64 to split (measured on
    the c1/c2 shapes: the 64-row FFN-out drops from 13.5 to 6-7 us; splitting
    c1's K = 256 projections too, whose residual sites then run their
    LayerNorm in the reduce kernel, takes c1 from 0.070 to 0.067 ms)."""
    tiles = -(-m // 128) * -(-n // 64)
    return 0 if k >= 256 and tiles * 4 < sms else None


# FFN row chunking (torch_transformer_benchmark.py:3841-3938): when the
# [rows, ffn_dim] hidden activation would take more than this fraction of the
# device's TOTAL memory (a hardware constant, so the decision is a pure
# function of shape and card, and needs no device sync inside a captured
# graph), FFN-in and FFN-out run over row chunks that reuse one hidden
# buffer. Each row of this build's GEMMs is computed independently with the
# same K order whatever the row count, so a chunked FFN is bit-identical to
# the unchunked one (the few-row split-K form, whose fixed-order sum of K
# parts rounds differently, only serves inputs thousands of times below the
# chunking threshold). On a 180 GB B200 the budget is ~34 GB; BASELINE's
# largest hidden (c4) is 2.1 GB, so c1-c5 never chunk.
FFN_CHUNK_BUDGET_FRAC = 3.0 / 16.0
FFN_CHUNK_MIN_ROWS = 256


def ffn_chunk_rows(rows: int, ffn_dim: int, elem_bytes: int, budget_bytes: int) -> Optional[int]:
    """Rows per FFN chunk, or None when the whole [rows, ffn_dim] hidden of
    `elem_bytes`-byte elements fits `budget_bytes`. Otherwise the largest
    power of two of rows whose hidden fits, but at least FFN_CHUNK_MIN_ROWS
    (the reference's floor, below which per-chunk launches dominate) and at
    most `rows` (torch_transformer_benchmark.py:3886-3908)."""
    if rows <= 0 or rows * ffn_dim * elem_bytes <= budget_bytes:
        return None
    fit = budget_bytes // max(ffn_dim * elem_bytes, 1)
    chunk = max(int(fit), FFN_CHUNK_MIN_ROWS)
    chunk = 1 << (chunk.bit_length() - 1)
    return min(chunk, rows)


class _GraphCacheEntry:
    """One captured forward: static input/mask, the graph and its output
    (torch_transformer_benchmark.py:2045-2068). `workspace` is the split-K
    workspace the graph's kernels were captured with (or None): the entry
    holds a reference so the caching allocator can never hand that memory to
    another tensor while the graph may still replay into it."""

    __slots__ = ("graph", "static_x", "static_mask", "static_output", "workspace")

    def __init__(self, graph, static_x, static_mask, static_output, workspace=None) -> None:
        self.graph = graph
        self.static_x = static_x
        self.static_mask = static_mask
        self.static_output = static_output
        self.workspace = workspace


# Captured graphs keep their working set alive in a private pool; above this
# fraction of device memory the forward stays eager (launch overhead is
# negligible for shapes that large anyway). Same policy as the reference's
# _graph_memory_safe (torch_transformer_benchmark.py:2489-2535), computed
# from this forward's own buffers.
_GRAPH_MEMORY_BUDGET_FRAC = 0.20


class UserOptimizedTransformer(BaselineTransformer):
    """Drop-in replacement of the reference's UserOptimizedTransformer
    (torch_transformer_benchmark.py:2144) on sm_100a kernels."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__(config)
        # plain attributes only: no parameters or buffers are added
        self._weights_key: Optional[Tuple] = None
        self._weights: Optional[list] = None
        self._final_ln: Optional[Tuple[torch.Tensor, torch.Tensor]] = None  # fp32 final LayerNorm w, b
        self._graph_cache: Dict[Tuple, _GraphCacheEntry] = {}
        self._graph_unsupported: set = set()
        self._graph_pool = None
        self._mask_all_true_cache: Dict[Tuple, bool] = {}
        self._splitk_ws: Optional[torch.Tensor] = None  # fp32 partials of split-K projections
        self._last_ws_used = False  # whether the last _forward_core used _splitk_ws
        self.use_cuda_graphs = True
        # FFN-out with split (hi/lo fp16) weights: twice that GEMM's tensor
        # work for a near-fp32 weight. None = automatic (deep stacks only,
        # where fp16 weight rounding accumulates over many residual adds).
        self.precise_ffn_out: Optional[bool] = None
        # bytes of hidden activation above which the FFN runs in row chunks;
        # None = FFN_CHUNK_BUDGET_FRAC of the device's total memory
        self.ffn_chunk_budget_bytes: Optional[int] = None
        # half-precision models: attention scores rounded as the eager model
        # in T rounds them, T(T(q . k) * scale) (torch_transformer_benchmark.py:
        # 173); False keeps fp32 scores (closer to the fp32 model, further
        # from eager T)
        self.round_half_scores = True
        # unsplit residual projections: the LayerNorm after each one starts on
        # the rows the GEMM has finished while its last wave still runs
        # (tf_gemm_residual_ready + tf_ln_ready); False runs it after the GEMM
        self.overlap_ln = True

    def _model_dtype(self) -> torch.dtype:
        return self.final_norm.weight.dtype

    def _split_ffn_out(self) -> bool:
        if self._model_dtype() != torch.float32:
            return False  # a half-precision model's weights are already in its own type
        if self.precise_ffn_out is not None:
            return bool(self.precise_ffn_out)
        return self.config.num_layers >= 16

    # ------------------------------------------------------------------ caches
    def _layer_weights(self) -> list:
        """Compute-type weight caches, rebuilt whenever a source parameter's
        storage, dtype or device changes (torch_transformer_benchmark.py:
        452-466)."""
        split = self._split_ffn_out()
        key = tuple((p.data_ptr(), p.dtype, p.device, p._version) for p in self.parameters()) + (split,)
        if self._weights is None or key != self._weights_key:
            ct = torch.bfloat16 if self._model_dtype() == torch.bfloat16 else torch.float16
            fn = self.final_norm
            self._weights = [_LayerWeights(blk, split, ct) for blk in self.layers]
            self._final_ln = (fn.weight.float().contiguous(), fn.bias.float().contiguous())
            self._weights_key = key
            self._graph_cache.clear()
        return self._weights

    def _resolve_mask_active(self, valid_token_mask: Optional[torch.Tensor]) -> bool:
        """Whether the mask disables any token: at most one device->host sync
        per distinct mask tensor (torch_transformer_benchmark.py:2438-2477)."""
        if valid_token_mask is None:
            return False
        try:
            version = valid_token_mask._version
        except RuntimeError:
            version = None
        key = (valid_token_mask.data_ptr(), tuple(valid_token_mask.shape), valid_token_mask.dtype, version)
        all_true = self._mask_all_true_cache.get(key)
        if all_true is None:
            all_true = bool(torch.all(valid_token_mask))
            self._mask_all_true_cache[key] = all_true
        return not all_true

    # ------------------------------------------------------------------ core
    def _forward_core(self, x: torch.Tensor, valid: Optional[torch.Tensor], mask_active: bool) -> torch.Tensor:
        """The per-layer schedule of torch_transformer_benchmark.py:4003-4326
        (fp16-GEMM branch 4130-4199). The residual adds of the reference's
        LayerNorm sites happen in the epilogues of out_proj and ffn_out
        (same masking points: mask_delta after attention, mask_x after the
        FFN); the LayerNorm kernels then only normalise. The residual stream is
        fp32 for the fp32 model and the model's type T for fp16/bf16 models
        (whose epilogues round the Linear output and the sum to T, and whose
        GELU reads the T-rounded Linear output). No host sync, so it is safe
        to capture."""
        cfg = self.config
        b, s, d = x.shape
        h = cfg.num_heads
        scale = (d // h) ** -0.5
        wts = self._layer_weights()
        vflat = valid.reshape(-1) if mask_active else None
        kvalid = valid if mask_active else None
        dev = x.device
        half = x.dtype != torch.float32
        ct = wts[0].wqkv.dtype  # compute (operand) type

        m, f = b * s, cfg.ffn_dim
        props = torch.cuda.get_device_properties(dev)
        budget = self.ffn_chunk_budget_bytes
        if budget is None:
            budget = int(props.total_memory * FFN_CHUNK_BUDGET_FRAC)
        chunk = ffn_chunk_rows(m, f, torch.finfo(ct).bits // 8, budget)

        x_res = torch.empty(b, s, d, dtype=x.dtype, device=dev)
        normed = torch.empty(b, s, d, dtype=ct, device=dev)
        qkv = torch.empty(b, s, 3 * d, dtype=ct, device=dev)
        ctx = torch.empty(b, s, d, dtype=ct, device=dev)
        hidden = torch.empty(b, s, f, dtype=ct, device=dev) if chunk is None else \
            torch.empty(chunk, f, dtype=ct, device=dev)

        # split-K (fp32 partials in a workspace) for the projections of
        # few-row inputs, where 128-row tiles would leave most SMs idle
        sms = props.multi_processor_count
        sk_qkv, sk_o, sk_1 = _splitk(m, 3 * d, d, sms), _splitk(m, d, d, sms), _splitk(m, f, d, sms)
        sk_2 = None if wts[0].split_w2 else _splitk(m, d, f, sms)
        ws = None
        if any(v is not None for v in (sk_qkv, sk_o, sk_1, sk_2)):
            need = max(kernels.splitk_workspace_bytes(m, n, k)
                       for n, k, v in ((3 * d, d, sk_qkv), (d, d, sk_o), (f, d, sk_1), (d, f, sk_2)) if v is not None)
            ws = self._splitk_ws
            if ws is None or ws.device != dev or ws.numel() < need:
                # a new tensor; graphs captured with the old one hold it alive
                # through their cache entries (_GraphCacheEntry.workspace)
                ws = self._splitk_ws = torch.empty(need, dtype=torch.uint8, device=dev)
        self._last_ws_used = ws is not None
        # per-8-row-group counters for the GEMM -> LayerNorm pairs that overlap
        # (zeroed here every forward, and by each LayerNorm as it consumes them)
        lno = self.overlap_ln and d <= 2048
        ready_o = lno and sk_o is None
        ready_2 = lno and sk_2 is None and chunk is None
        ready = kernels.ready_counters(m, dev) if (ready_o or ready_2) else None

        # With split-K residual projections (few rows), their reduce kernel also
        # runs the LayerNorm that follows (the next layer's norm1, or the final
        # norm after the last layer): one launch fewer per residual site.
        cur = x  # residual stream; the caller's x is read, never written
        out = None
        normed_ready = False  # normed already holds this layer's norm1 output
        n_layers = len(self.layers)
        for li, blk in enumerate(self.layers):
            w = wts[li]
            if not normed_ready:
                kernels.ln_residual(cur, None, w.n1w, w.n1b, blk.norm1.eps, normed=normed)
            kernels.linear(normed, w.wqkv, w.bqkv, out=qkv, splits=sk_qkv, workspace=ws)
            kernels.flash_attention(qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:], h, scale,
                                    causal=cfg.causal, key_valid=kvalid, out=ctx,
                                    round_scores=half and self.round_half_scores)
            if sk_o is not None:
                cur, _ = kernels.linear_residual_ln(ctx, w.wo, w.bo, cur, x_res, vflat, w.n2w, w.n2b,
                                                    blk.norm2.eps, mask_delta=mask_active, normed=normed,
                                                    splits=sk_o, workspace=ws)
            elif ready_o:
                cur = kernels.linear_residual(ctx, w.wo, w.bo, cur, x_res, vflat, mask_delta=mask_active,
                                              ready=ready)
                kernels.ln_ready(cur, w.n2w, w.n2b, blk.norm2.eps, ready, normed=normed)
            else:
                cur = kernels.linear_residual(ctx, w.wo, w.bo, cur, x_res, vflat, mask_delta=mask_active)
                kernels.ln_residual(cur, None, w.n2w, w.n2b, blk.norm2.eps, normed=normed)
            if chunk is not None:
                # row-chunked FFN (cur is x_res here, updated in place)
                n2, c2 = normed.view(m, d), cur.view(m, d)
                for r0 in range(0, m, chunk):
                    r1 = min(m, r0 + chunk)
                    hc = hidden[:r1 - r0]
                    kernels.linear(n2[r0:r1], w.w1, w.b1, gelu=True, out=hc, round_gelu_input=half)
                    kernels.linear_residual(hc, w.w2, w.b2, c2[r0:r1], c2[r0:r1],
                                            vflat[r0:r1] if vflat is not None else None, mask_x=mask_active,
                                            w_split=w.split_w2)
                normed_ready = False
                continue
            kernels.linear(normed, w.w1, w.b1, gelu=True, out=hidden, splits=sk_1, workspace=ws,
                           round_gelu_input=half)
            if sk_2 is None and ready_2:
                cur = kernels.linear_residual(hidden, w.w2, w.b2, cur, x_res, vflat, mask_x=mask_active,
                                              w_split=w.split_w2, ready=ready)
                if li + 1 < n_layers:
                    wn, nxt = wts[li + 1], self.layers[li + 1]
                    kernels.ln_ready(cur, wn.n1w, wn.n1b, nxt.norm1.eps, ready, normed=normed)
                    normed_ready = True
                else:
                    fw, fb = self._final_ln
                    out = kernels.ln_ready(cur, fw, fb, self.final_norm.eps, ready, vflat, mask_out=mask_active,
                                           out_dtype=x.dtype)
            elif sk_2 is None:
                kernels.linear_residual(hidden, w.w2, w.b2, cur, x_res, vflat, mask_x=mask_active,
                                        w_split=w.split_w2)
                normed_ready = False
            elif li + 1 < n_layers:
                wn, nxt = wts[li + 1], self.layers[li + 1]
                kernels.linear_residual_ln(hidden, w.w2, w.b2, cur, x_res, vflat, wn.n1w, wn.n1b, nxt.norm1.eps,
                                           mask_x=mask_active, normed=normed, splits=sk_2, workspace=ws)
                normed_ready = True
            else:
                fw, fb = self._final_ln
                _, out = kernels.linear_residual_ln(hidden, w.w2, w.b2, cur, x_res, vflat, fw, fb,
                                                    self.final_norm.eps, mask_x=mask_active, mask_out=mask_active,
                                                    out_dtype=x.dtype, splits=sk_2, workspace=ws)
        if out is None:
            fw, fb = self._final_ln
            _, out = kernels.ln_residual(cur, None, fw, fb, self.final_norm.eps, vflat, mask_out=mask_active,
                                         out_dtype=x.dtype)
        return out

    # ------------------------------------------------------------------ graphs
    def _graph_memory_safe(self, x: torch.Tensor) -> bool:
        b, s, d = x.shape
        m = b * s
        per_row = 4 * d * 3 + 2 * (d * 6 + self.config.ffn_dim)  # x_res, out, static_x + fp16 buffers
        total = torch.cuda.get_device_properties(x.device).total_memory
        return m * per_row <= int(total * _GRAPH_MEMORY_BUDGET_FRAC)

    def _capture_graph(self, x, valid, mask_active) -> _GraphCacheEntry:
        """Capture the whole forward once per key: 3 warm-up runs on a side
        stream, then capture into a shared pool
        (torch_transformer_benchmark.py:3648-3725)."""
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        static_x = x.clone()
        static_mask = valid.clone() if mask_active else None
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                self._forward_core(static_x, static_mask, mask_active)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._graph_pool):
            static_out = self._forward_core(static_x, static_mask, mask_active)
        # the workspace the captured kernels write (None when no projection of
        # this shape is split): a later, larger shape replaces
        # self._splitk_ws, and this reference keeps the old one alive
        ws = self._splitk_ws if self._last_ws_used else None
        return _GraphCacheEntry(graph, static_x, static_mask, static_out, ws)

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        cfg = self.config
        if not x.is_cuda:
            raise RuntimeError("UserOptimizedTransformer needs a CUDA (B200) tensor; there is no CPU path")
        if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise NotImplementedError(f"input dtype {x.dtype}: fp32, fp16 and bf16 models are implemented")
        if self._model_dtype() != x.dtype:
            raise ValueError(f"x is {x.dtype} but the model's parameters are {self._model_dtype()}: convert both "
                             "to one dtype (model.to(dtype) and x.to(dtype))")
        if x.dim() != 3 or x.shape[-1] != cfg.d_model:
            raise ValueError(f"expected x of shape [B, S, {cfg.d_model}], got {tuple(x.shape)}")
        if not x.is_contiguous():
            x = x.contiguous()
        if valid_token_mask is not None:
            if valid_token_mask.shape != x.shape[:2]:
                raise ValueError("valid_token_mask must be [B, S]")
            if valid_token_mask.dtype != torch.bool:
                valid_token_mask = valid_token_mask.bool()
        mask_active = self._resolve_mask_active(valid_token_mask)
        mask_kind = "none" if valid_token_mask is None else ("partial" if mask_active else "all_true")

        if not self.use_cuda_graphs or not self._graph_memory_safe(x):
            return self._forward_core(x, valid_token_mask, mask_active)
        key = (tuple(x.shape), x.dtype, x.device, cfg.causal, mask_kind, self._split_ffn_out(),
               self.ffn_chunk_budget_bytes, self.round_half_scores, self.overlap_ln)
        if key in self._graph_unsupported:
            return self._forward_core(x, valid_token_mask, mask_active)
        self._layer_weights()  # may invalidate cached graphs
        entry = self._graph_cache.get(key)
        if entry is None:
            try:
                entry = self._capture_graph(x, valid_token_mask, mask_active)
            except Exception:
                # capture failed: this key runs the same kernels eagerly from now on
                self._graph_unsupported.add(key)
                return self._forward_core(x, valid_token_mask, mask_active)
            self._graph_cache[key] = entry
        entry.static_x.copy_(x)
        if mask_active:
            entry.static_mask.copy_(valid_token_mask)
        entry.graph.replay()
        return entry.static_output.clone()
