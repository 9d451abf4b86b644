"""Tensor-level wrappers over the C ABI (one per exported kernel).

Each wrapper checks dtypes, devices and strides, allocates its output when
the caller gives none, and enqueues the kernel on the current CUDA stream
(so it can be captured in a CUDA graph). None of them has a fallback: a
tensor on the CPU, a wrong dtype or a missing library raises.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _abi


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(name: str, *ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{name}: every operand must be a CUDA tensor (no CPU path)")


HALF_TYPES = (torch.float16, torch.bfloat16)


def ln_residual(x: torch.Tensor, delta: Optional[torch.Tensor], weight: torch.Tensor, bias: torch.Tensor,
                eps: float, valid: Optional[torch.Tensor] = None, *, mask_delta: bool = False,
                mask_x: bool = False, mask_out: bool = False, write_x: bool = False,
                x_out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                normed: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """One residual site (tf_ln_residual). x: fp32 [..., D] contiguous with
    delta fp16 of the same shape or None (the fp32 model), or x fp16/bf16 with
    delta of x's type (a half-precision model: x + delta is rounded to that
    type); weight and bias fp32; valid: bool/uint8 [rows] or None. normed is
    fp16 (fp32 x) or x's type (half x) unless out_dtype is fp32.
    Returns (x_new, normed); x_new is x_out (may be x itself: the kernel reads
    each row fully before writing it) when write_x, else x."""
    _need_cuda("ln_residual", x, delta, weight, bias, valid, x_out, normed)
    if x.dtype not in (torch.float32,) + HALF_TYPES or not x.is_contiguous():
        raise ValueError("ln_residual: x must be contiguous fp32, fp16 or bf16")
    half = x.dtype in HALF_TYPES
    d = x.shape[-1]
    m = x.numel() // d
    delta_dtype = x.dtype if half else torch.float16
    if delta is not None and (delta.dtype != delta_dtype or not delta.is_contiguous() or delta.numel() != x.numel()):
        raise ValueError(f"ln_residual: delta must be contiguous {delta_dtype} shaped like x")
    if weight.dtype != torch.float32 or bias.dtype != torch.float32:
        raise ValueError("ln_residual: weight and bias must be fp32")
    flags = 0
    if mask_delta:
        flags |= _abi.TF_LN_MASK_DELTA
    if mask_x:
        flags |= _abi.TF_LN_MASK_X
    if mask_out:
        flags |= _abi.TF_LN_MASK_OUT
    if flags and (valid is None or valid.numel() != m):
        raise ValueError("ln_residual: masking needs a valid-token mask with one entry per row")
    if valid is not None and valid.dtype not in (torch.bool, torch.uint8):
        raise ValueError("ln_residual: valid must be bool or uint8")
    if valid is not None and not valid.is_contiguous():
        valid = valid.contiguous()
    if write_x:
        flags |= _abi.TF_LN_WRITE_X
        if x_out is None:
            x_out = torch.empty_like(x)
    if x.dtype == torch.float16:
        flags |= _abi.TF_LN_X_F16
    elif x.dtype == torch.bfloat16:
        flags |= _abi.TF_LN_X_BF16
    if out_dtype is None:
        out_dtype = x.dtype if half else torch.float16
    if out_dtype == torch.float32:
        flags |= _abi.TF_LN_OUT_F32
    elif out_dtype != delta_dtype:
        raise ValueError(f"ln_residual: out_dtype must be {delta_dtype} or fp32")
    if normed is None:
        normed = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    _abi.call("tf_ln_residual", _ptr(x), _ptr(delta), _ptr(weight), _ptr(bias), float(eps),
              _ptr(valid) if flags & 7 else None, m, d, flags, _ptr(x_out), _ptr(normed), _stream())
    return (x_out if write_x else x), normed


def ready_counters(rows: int, device) -> torch.Tensor:
    """Zeroed counters for a linear_residual / ln_ready pair: one per 8-row
    group, then the LayerNorm's two ticket counters."""
    return torch.zeros((rows + 7) // 8 + 2, dtype=torch.int32, device=device)


def _check_ready(ready: torch.Tensor, rows: int, name: str) -> None:
    if ready.dtype != torch.int32 or not ready.is_contiguous() or ready.numel() < (rows + 7) // 8 + 2:
        raise ValueError(f"{name}: ready must be contiguous int32 with ceil(rows / 8) + 2 entries")


def ln_ready(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float, ready: torch.Tensor,
             valid: Optional[torch.Tensor] = None, *, mask_out: bool = False,
             out_dtype: Optional[torch.dtype] = None, normed: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm of x while the linear_residual(..., ready=ready) launched just
    before it on this stream is still storing x (tf_ln_ready): each 8-row group
    is normalised once its count reaches D, and its count is reset to 0.
    normed = mask_out(LayerNorm(x) * weight + bias), fp16 (fp32 x) or x's type
    (half x) unless out_dtype is fp32. D <= 2048."""
    _need_cuda("ln_ready", x, weight, bias, ready, valid, normed)
    if x.dtype not in (torch.float32,) + HALF_TYPES or not x.is_contiguous():
        raise ValueError("ln_ready: x must be contiguous fp32, fp16 or bf16")
    if weight.dtype != torch.float32 or bias.dtype != torch.float32:
        raise ValueError("ln_ready: weight and bias must be fp32")
    half = x.dtype in HALF_TYPES
    d = x.shape[-1]
    m = x.numel() // d
    _check_ready(ready, m, "ln_ready")
    flags = 0
    if mask_out:
        if valid is None or valid.numel() != m or valid.dtype not in (torch.bool, torch.uint8):
            raise ValueError("ln_ready: mask_out needs a bool/uint8 mask with one entry per row")
        valid = valid.contiguous()
        flags |= _abi.TF_LN_MASK_OUT
    if x.dtype == torch.float16:
        flags |= _abi.TF_LN_X_F16
    elif x.dtype == torch.bfloat16:
        flags |= _abi.TF_LN_X_BF16
    io_dtype = x.dtype if half else torch.float16
    if out_dtype is None:
        out_dtype = io_dtype
    if out_dtype == torch.float32:
        flags |= _abi.TF_LN_OUT_F32
    elif out_dtype != io_dtype:
        raise ValueError(f"ln_ready: out_dtype must be {io_dtype} or fp32")
    if normed is None:
        normed = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    _abi.call("tf_ln_ready", _ptr(x), _ptr(weight), _ptr(bias), float(eps), _ptr(valid) if mask_out else None,
              m, d, flags, _ptr(normed), _ptr(ready), _stream())
    return normed


def _gemm_operands(name, a, w, b, w_split):
    _need_cuda(name, a, w, b)
    if a.dtype not in HALF_TYPES or w.dtype != a.dtype:
        raise ValueError(f"{name}: a and w must both be fp16 or both bf16")
    if w_split and a.dtype != torch.float16:
        raise ValueError(f"{name}: split weights are fp16")
    if b.dtype != torch.float32 or not b.is_contiguous():
        raise ValueError(f"{name}: bias must be contiguous fp32")
    k = a.shape[-1]
    n = w.shape[0]
    if w.shape[1] != (2 * k if w_split else k) or b.numel() != n:
        raise ValueError(f"{name}: weight must be [N, {'2K' if w_split else 'K'}] and bias [N]")
    a2 = a.reshape(-1, k)
    if a2.stride(-1) != 1 or w.stride(-1) != 1:
        raise ValueError(f"{name}: operands need a unit inner stride")
    return a2, n, k


def split_weight(w: torch.Tensor) -> torch.Tensor:
    """[N, K] fp32 weight -> [N, 2K] fp16 [W_hi | W_lo] with W_hi = fp16(W),
    W_lo = fp16(W - W_hi): the pair represents W to ~2^-22 relative."""
    w = w.detach().float()
    hi = w.half()
    lo = (w - hi.float()).half()
    return torch.cat([hi, lo], dim=1).contiguous()


def splitk_workspace_bytes(m: int, n: int, k: int, splits: int = 0) -> int:
    """Bytes of fp32 partial sums a split-K call of this shape needs
    (tf_gemm_splitk_workspace; splits 0 = automatic)."""
    _abi.load()
    return int(_abi.call_value("tf_gemm_splitk_workspace", int(m), int(n), int(k), int(splits)))


def _splitk_ws(workspace: Optional[torch.Tensor], m: int, n: int, k: int, splits: int, device) -> torch.Tensor:
    need = splitk_workspace_bytes(m, n, k, splits)
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=device)
    _need_cuda("split-K workspace", workspace)
    if workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"split-K workspace of {need} bytes needed")
    return workspace


def linear(a: torch.Tensor, w: torch.Tensor, b: torch.Tensor, *, gelu: bool = False,
           out: Optional[torch.Tensor] = None, tile_n: int = 0, w_split: bool = False,
           pair: int = 0, splits: Optional[int] = None, workspace: Optional[torch.Tensor] = None,
           round_gelu_input: bool = False) -> torch.Tensor:
    """16-bit GEMM on tcgen05 (tf_gemm): out = T([gelu](a @ w.T + b)) with T
    = a's type, a [..., K] fp16 or bf16 with unit inner stride, w [N, K] of
    the same type (or split_weight's fp16 [N, 2K] with w_split), b [N] fp32.
    round_gelu_input: GELU of T(a @ w.T + b), as F.gelu applied to a stored
    Linear output of a half-precision model. splits (0 = automatic) selects
    the split-K form (tf_gemm_splitk) with `workspace` (allocated if None)."""
    a2, n, k = _gemm_operands("linear", a, w, b, w_split)
    _need_cuda("linear", out)
    m = a2.shape[0]
    if out is None:
        out = torch.empty(*a.shape[:-1], n, dtype=a.dtype, device=a.device)
    o2 = out.view(-1, n) if out.is_contiguous() else out
    if o2.stride(-1) != 1 or o2.dtype != a.dtype:
        raise ValueError("linear: out must have a's type and a unit inner stride")
    epi = _abi.TF_EPI_BIAS
    if gelu:
        epi = _abi.TF_EPI_BIAS_GELU_ROUNDED if round_gelu_input else _abi.TF_EPI_BIAS_GELU
    if a.dtype == torch.bfloat16:
        epi |= _abi.TF_EPI_BF16
    if splits is not None:
        if w_split:
            raise ValueError("linear: split-K does not take split weights")
        ws = _splitk_ws(workspace, m, n, k, splits, a.device)
        _abi.call("tf_gemm_splitk", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(o2), o2.stride(0),
                  m, n, k, epi, int(splits), _ptr(ws), ws.numel() * ws.element_size(), _stream())
        return out
    epi |= _abi.TF_EPI_W_SPLIT if w_split else 0
    if tile_n or pair:
        _abi.call("tf_gemm_tiled", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(o2), o2.stride(0),
                  m, n, k, epi, tile_n, pair, _stream())
    else:
        _abi.call("tf_gemm", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(o2), o2.stride(0),
                  m, n, k, epi, _stream())
    return out


def linear_residual(a: torch.Tensor, w: torch.Tensor, b: torch.Tensor, x_in: torch.Tensor,
                    x_out: Optional[torch.Tensor] = None, valid: Optional[torch.Tensor] = None, *,
                    mask_delta: bool = False, mask_x: bool = False, w_split: bool = False, tile_n: int = 0,
                    pair: int = 0, splits: Optional[int] = None,
                    workspace: Optional[torch.Tensor] = None, ready: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GEMM closing a residual connection (tf_gemm_residual):
    x_out = mask_x(x_in + mask_delta(a @ w.T + b)). x_in/x_out [..., N]
    contiguous (x_out may be x_in), fp32, or a's type for a half-precision
    model (then both the Linear's output and the sum are rounded to it, as the
    eager model stores them); valid bool/uint8 [rows] for the masks.
    splits (0 = automatic) selects tf_gemm_residual_splitk. ready (int32
    [ceil(rows / 8) + 2], zero, from ready_counters) selects
    tf_gemm_residual_ready: the epilogue counts the stored columns per 8-row
    group for an ln_ready launched right after it."""
    a2, n, k = _gemm_operands("linear_residual", a, w, b, w_split)
    _need_cuda("linear_residual", x_in, x_out, valid)
    if x_in.dtype not in (torch.float32, a.dtype) or not x_in.is_contiguous() or x_in.shape[-1] != n:
        raise ValueError("linear_residual: x_in must be contiguous fp32 or a's type [..., N]")
    if x_out is None:
        x_out = torch.empty_like(x_in)
    if x_out.shape != x_in.shape or x_out.dtype != x_in.dtype or not x_out.is_contiguous():
        raise ValueError("linear_residual: x_out must match x_in")
    m = a2.shape[0]
    if x_in.numel() // n != m:
        raise ValueError("linear_residual: row count of a and x differ")
    if mask_delta and mask_x:
        raise ValueError("linear_residual: one mask mode at a time")
    mode = _abi.TF_RES_MASK_DELTA if mask_delta else (_abi.TF_RES_MASK_X if mask_x else _abi.TF_RES_NO_MASK)
    if mode and (valid is None or valid.numel() != m or valid.dtype not in (torch.bool, torch.uint8)):
        raise ValueError("linear_residual: masking needs a bool/uint8 mask with one entry per row")
    opts = (_abi.TF_RES_X16 if x_in.dtype != torch.float32 else 0) | (
        _abi.TF_RES_BF16 if a.dtype == torch.bfloat16 else 0)
    if valid is not None and not valid.is_contiguous():
        valid = valid.contiguous()
    if ready is not None:
        _need_cuda("linear_residual", ready)
        if splits is not None or tile_n or pair:
            raise ValueError("linear_residual: ready counters take the automatic, unsplit tiling")
        _check_ready(ready, m, "linear_residual")
        _abi.call("tf_gemm_residual_ready", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(x_in),
                  _ptr(x_out), n, _ptr(valid) if mode else None, mode | opts, m, n, k, 1 if w_split else 0,
                  _ptr(ready), _stream())
        return x_out
    if splits is not None:
        if w_split:
            raise ValueError("linear_residual: split-K does not take split weights")
        ws = _splitk_ws(workspace, m, n, k, splits, a.device)
        _abi.call("tf_gemm_residual_splitk", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(x_in),
                  _ptr(x_out), n, _ptr(valid) if mode else None, mode | opts, m, n, k, int(splits), _ptr(ws),
                  ws.numel() * ws.element_size(), _stream())
        return x_out
    _abi.call("tf_gemm_residual", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(x_in), _ptr(x_out), n,
              _ptr(valid) if mode else None, mode | opts, m, n, k, 1 if w_split else 0, tile_n, pair, _stream())
    return x_out


def linear_residual_ln(a: torch.Tensor, w: torch.Tensor, b: torch.Tensor, x_in: torch.Tensor,
                       x_out: Optional[torch.Tensor], valid: Optional[torch.Tensor], ln_weight: torch.Tensor,
                       ln_bias: torch.Tensor, eps: float, *, mask_delta: bool = False, mask_x: bool = False,
                       mask_out: bool = False, normed: Optional[torch.Tensor] = None,
                       out_dtype: Optional[torch.dtype] = None, splits: int = 0,
                       workspace: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Split-K residual projection whose reduce kernel also runs the
    LayerNorm of the result (tf_gemm_residual_ln_splitk): x_out as
    linear_residual, normed = mask_out(LayerNorm(x_out) * ln_weight +
    ln_bias). normed is fp16 (fp32 x) or x's type (half x) unless out_dtype
    is fp32. Returns (x_out, normed)."""
    a2, n, k = _gemm_operands("linear_residual_ln", a, w, b, False)
    _need_cuda("linear_residual_ln", x_in, x_out, valid, ln_weight, ln_bias, normed)
    if x_in.dtype not in (torch.float32, a.dtype) or not x_in.is_contiguous() or x_in.shape[-1] != n:
        raise ValueError("linear_residual_ln: x_in must be contiguous fp32 or a's type [..., N]")
    if x_out is None:
        x_out = torch.empty_like(x_in)
    if x_out.shape != x_in.shape or x_out.dtype != x_in.dtype or not x_out.is_contiguous():
        raise ValueError("linear_residual_ln: x_out must match x_in")
    m = a2.shape[0]
    if x_in.numel() // n != m:
        raise ValueError("linear_residual_ln: row count of a and x differ")
    if mask_delta and mask_x:
        raise ValueError("linear_residual_ln: one mask mode at a time")
    if ln_weight.dtype != torch.float32 or ln_bias.dtype != torch.float32 or ln_weight.numel() != n:
        raise ValueError("linear_residual_ln: LayerNorm weight and bias must be fp32 [N]")
    mode = _abi.TF_RES_MASK_DELTA if mask_delta else (_abi.TF_RES_MASK_X if mask_x else _abi.TF_RES_NO_MASK)
    if (mode or mask_out) and (valid is None or valid.numel() != m or valid.dtype not in (torch.bool, torch.uint8)):
        raise ValueError("linear_residual_ln: masking needs a bool/uint8 mask with one entry per row")
    if valid is not None and not valid.is_contiguous():
        valid = valid.contiguous()
    half = x_in.dtype != torch.float32
    if out_dtype is None:
        out_dtype = x_in.dtype if half else torch.float16
    if out_dtype not in (torch.float32, x_in.dtype if half else torch.float16):
        raise ValueError("linear_residual_ln: out_dtype must be fp32 or the 16-bit type of the stream")
    if normed is None:
        normed = torch.empty(x_in.shape, dtype=out_dtype, device=x_in.device)
    if normed.shape != x_in.shape or normed.dtype != out_dtype or not normed.is_contiguous():
        raise ValueError("linear_residual_ln: normed must be contiguous, shaped like x, of out_dtype")
    opts = (_abi.TF_RES_X16 if half else 0) | (_abi.TF_RES_BF16 if a.dtype == torch.bfloat16 else 0)
    ln_flags = (_abi.TF_LN_MASK_OUT if mask_out else 0) | (_abi.TF_LN_OUT_F32 if out_dtype == torch.float32 else 0)
    ws = _splitk_ws(workspace, m, n, k, splits, a.device)
    use_valid = mode or mask_out
    _abi.call("tf_gemm_residual_ln_splitk", _ptr(a2), a2.stride(0), _ptr(w), w.stride(0), _ptr(b), _ptr(x_in),
              _ptr(x_out), n, _ptr(valid) if use_valid else None, mode | opts, m, n, k, int(splits), _ptr(ws),
              ws.numel() * ws.element_size(), _ptr(ln_weight), _ptr(ln_bias), float(eps), _ptr(normed), ln_flags,
              _stream())
    return x_out, normed


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float, *,
                    causal: bool = False, key_valid: Optional[torch.Tensor] = None, q_pos0: int = 0,
                    k_pos0: int = 0, out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                    lse: Optional[torch.Tensor] = None, want_lse: bool = False, exp_f16x2: bool = False,
                    fma_exp_pairs: int = 0, round_scores: bool = False):
    """Flash attention forward (tf_flash_fwd).

    q: [B, Sq, H*hd] fp16 or bf16 view with unit inner stride (may be a
    column slice of a packed QKV buffer), k, v: [B, Sk, H*hd] likewise, of
    q's type. Returns out [B, Sq, H*hd] (q's type unless out_dtype is fp32)
    and, with want_lse or an lse buffer, the natural-log sum-exp [B, H, Sq]
    fp32. round_scores: the scores of the eager model in q's type,
    T(T(q . k) * scale), before the fp32 softmax (half-precision models)."""
    _need_cuda("flash_attention", q, k, v, key_valid, out, lse)
    for t in (q, k, v):
        if t.dtype not in HALF_TYPES or t.dtype != q.dtype or t.dim() != 3 or t.stride(-1) != 1:
            raise ValueError("flash_attention: q, k, v must be fp16 or bf16 [B, S, H*hd] (one type) with unit "
                             "inner stride")
    if out_dtype is None:
        out_dtype = q.dtype
    if out_dtype not in (q.dtype, torch.float32):
        raise ValueError("flash_attention: out_dtype must be q's type or fp32")
    bsz, sq, dq = q.shape
    sk = k.shape[1]
    if k.shape != v.shape or k.shape[0] != bsz or k.shape[2] != dq or v.stride() != k.stride():
        raise ValueError("flash_attention: k and v must have matching shapes and strides")
    if dq % heads:
        raise ValueError("flash_attention: feature width not divisible by heads")
    hd = dq // heads
    if out is None:
        out = torch.empty(bsz, sq, dq, dtype=out_dtype, device=q.device)
    if out.stride(-1) != 1 or out.dtype != out_dtype:
        raise ValueError("flash_attention: out must match out_dtype with unit inner stride")
    if lse is None and want_lse:
        lse = torch.empty(bsz, heads, sq, dtype=torch.float32, device=q.device)
    if key_valid is not None:
        if key_valid.shape != (bsz, sk) or key_valid.dtype not in (torch.bool, torch.uint8):
            raise ValueError("flash_attention: key_valid must be bool [B, Sk]")
        key_valid = key_valid.contiguous()
    flags = (_abi.TF_ATTN_CAUSAL if causal else 0) | (_abi.TF_ATTN_OUT_F32 if out_dtype == torch.float32 else 0)
    if q.dtype == torch.bfloat16:
        flags |= _abi.TF_ATTN_BF16
    if exp_f16x2:
        flags |= _abi.TF_ATTN_EXP_F16X2
    if round_scores:
        flags |= _abi.TF_ATTN_ROUND_SCORES
    flags |= (int(fma_exp_pairs) & 0xFF) << 8
    _abi.call("tf_flash_fwd", _ptr(q), _ptr(k), _ptr(v), q.stride(1), k.stride(1), q.stride(0), k.stride(0),
              _ptr(out), out.stride(1), out.stride(0), _ptr(lse), _ptr(key_valid), bsz, heads, sq, sk, hd,
              float(scale), int(q_pos0), int(k_pos0), flags, _stream())
    return out, lse


def attn_merge(o_acc: torch.Tensor, lse_acc: torch.Tensor, o_part: torch.Tensor, lse_part: torch.Tensor,
               heads: int, out16: Optional[torch.Tensor] = None) -> None:
    """Merge a partial attention result into a running one in place
    (tf_attn_merge); optionally also write the merged result as fp16."""
    _need_cuda("attn_merge", o_acc, lse_acc, o_part, lse_part, out16)
    for t in (o_acc, o_part, lse_acc, lse_part):
        if t.dtype != torch.float32:
            raise ValueError("attn_merge: accumulators must be fp32")
    if o_acc.stride() != o_part.stride() or o_acc.shape != o_part.shape:
        raise ValueError("attn_merge: o_acc and o_part must share shape and strides")
    if not (lse_acc.is_contiguous() and lse_part.is_contiguous()):
        raise ValueError("attn_merge: lse tensors must be contiguous")
    bsz, sq, dq = o_acc.shape
    ld16 = out16.stride(1) if out16 is not None else 0
    bs16 = out16.stride(0) if out16 is not None else 0
    _abi.call("tf_attn_merge", _ptr(o_acc), _ptr(lse_acc), _ptr(o_part), _ptr(lse_part), o_acc.stride(1),
              o_acc.stride(0), _ptr(out16), ld16, bs16, bsz, heads, sq, dq // heads, _stream())


def wait_timeout_probe(src: torch.Tensor, limit_ns: int) -> torch.Tensor:
    """Run the bounded-wait probe (tf_test_wait_timeout): a wait that nothing
    completes runs out after limit_ns and records device code 106; the probe
    drains its own 4 KiB copy from `src` and returns. Returns the int32[3]
    result (timed out, drained, last byte copied) on the device."""
    _need_cuda("wait_timeout_probe", src)
    if src.numel() * src.element_size() < 4096 or not src.is_contiguous():
        raise ValueError("wait_timeout_probe: src must be contiguous with at least 4096 bytes")
    out = torch.full((3,), -7, dtype=torch.int32, device=src.device)
    _abi.call("tf_test_wait_timeout", _ptr(src), int(limit_ns), _ptr(out), _stream())
    return out
