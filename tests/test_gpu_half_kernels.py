"""Kernel-level parity of the half-precision model path on a B200: the fp16
and bf16 forms of each kernel (C ABI flags TF_LN_X_F16/BF16, TF_EPI_BF16,
TF_EPI_BIAS_GELU_ROUNDED, TF_RES_X16/BF16, TF_ATTN_BF16) against the oracle's
statement of the eager model's roundings in that type (oracle/
reference_model.py: ln_site_half, linear_half, linear_residual_half,
attention_fp16), on seeded inputs.

Tolerances (written per test; U = 2^-10 for fp16 and 2^-7 for bf16, one unit
in the last place relative to the value):
* LayerNorm: the stored sum x + delta is exact (the same single rounding);
  normed within one ulp of the fp32 LayerNorm of it: |d| <= U*|ref| + 1e-6.
* GEMM: the fp32 accumulation (error below 2^-20 * sum|a_i w_i| =: E) may
  tip the one rounding of the exact sum: |d| <= U*|ref| + E + 1e-6.
* GELU of the stored Linear output: its input may sit one ulp (+E) off, and
  the GELU slope is below 1.13: |d| <= U*(1.13*|h| + |ref|) + 1.13*E + 1e-6.
* residual in T: the stored projection v and then the sum may each be one
  ulp off: |d| <= U*(|v| + |ref|) + E + 1e-6.
* attention (bf16): P is rounded to bf16 before the PV product and the
  output to bf16: |d| <= 2e-2*|ref| + 4e-3 against fp32 attention of the same
  bf16 operands.
"""

import pytest
import torch

from oracle import reference_model as om

pytestmark = pytest.mark.gpu

TYPES = [torch.float16, torch.bfloat16]
ULP = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}


@pytest.fixture(scope="module")
def K():
    from transformer_optimization_b200 import _abi, kernels
    _abi.load()
    torch.backends.cuda.matmul.allow_tf32 = False
    yield kernels
    assert _abi.device_status() == 0, "a kernel wait ran out"


def _name(t):
    return "bf16" if t == torch.bfloat16 else "fp16"


def _acc_err(a, w):
    """Bound on the fp32 accumulation error of a @ w.T: 2^-20 * sum |a_i w_i|."""
    return 2.0 ** -20 * (a.double().abs() @ w.double().abs().t()).float()


def _assert_within(out, ref, bound, what):
    d = (out.float().cpu() - ref).abs()
    bad = d > bound
    assert not bool(bad.any()), (f"{what}: {int(bad.sum())}/{d.numel()} beyond bound, worst excess "
                                 f"{float((d - bound).max()):.3g}")


@pytest.mark.parametrize("dt", TYPES, ids=_name)
@pytest.mark.parametrize("m,d", [(7, 64), (1000, 1024), (333, 2048), (40, 4096), (148 * 8 * 6 + 3, 1024)])
@pytest.mark.parametrize("flags", ["plain", "delta", "mask_delta", "mask_x", "final"])
def test_ln_half(K, dt, m, d, flags):
    g = torch.Generator().manual_seed(m * 31 + d + len(flags))
    x = (torch.randn(m, d, generator=g) * 2 + 0.5).to(dt)
    delta = (torch.randn(m, d, generator=g) * 0.5).to(dt)
    w = torch.randn(d, generator=g) * 0.1 + 1
    b = torch.randn(d, generator=g) * 0.1
    valid = torch.rand(m, generator=g) > 0.3
    use_delta = flags != "plain"
    md, mx, mo = flags == "mask_delta", flags in ("mask_x", "final"), flags == "final"
    out_f32 = flags == "final"
    xr, yr = om.ln_site_half(x, delta if use_delta else None, w, b, 1e-5, valid, md, mx, mo, dt)
    dv = torch.device("cuda:0")
    x_new, y = K.ln_residual(x.to(dv), delta.to(dv) if use_delta else None, w.to(dv), b.to(dv), 1e-5,
                             valid.to(dv), mask_delta=md, mask_x=mx, mask_out=mo, write_x=use_delta,
                             out_dtype=torch.float32 if out_f32 else dt)
    torch.cuda.synchronize()
    assert y.dtype == (torch.float32 if out_f32 else dt)
    if use_delta:
        assert x_new.dtype == dt
        assert torch.equal(x_new.float().cpu(), xr)  # the same one rounding of x + delta
    if out_f32:
        assert torch.allclose(y.cpu(), yr, atol=2e-5, rtol=1e-5)
    else:
        _assert_within(y, yr, ULP[dt] * yr.abs() + 1e-6, "normed")


@pytest.mark.parametrize("dt", TYPES, ids=_name)
@pytest.mark.parametrize("m,n,k,kw", [
    (300, 256, 192, {}),                          # ragged rows, 1-CTA tiles
    (4096, 1024, 512, {}),                        # 2-SM pair tiles
    (2048, 384, 256, {"tile_n": 128, "pair": 1}),
    (64, 512, 2048, {"splits": 0}),               # split-K (few rows)
])
@pytest.mark.parametrize("gelu", [False, True])
def test_linear_half(K, dt, m, n, k, kw, gelu):
    g = torch.Generator().manual_seed(m + n + k + gelu)
    a = torch.randn(m, k, generator=g).to(dt)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dt)
    b = torch.randn(n, generator=g) * 0.1
    ref = om.linear_half(a, w, b, gelu, dt)
    dv = torch.device("cuda:0")
    out = K.linear(a.to(dv), w.to(dv), b.to(dv), gelu=gelu, round_gelu_input=gelu, **kw)
    torch.cuda.synchronize()
    assert out.dtype == dt
    e = _acc_err(a, w)
    if gelu:
        h = om.linear_half(a, w, b, False, dt)
        bound = ULP[dt] * (1.13 * h.abs() + ref.abs()) + 1.13 * e + 1e-6
    else:
        bound = ULP[dt] * ref.abs() + e + 1e-6
    _assert_within(out, ref, bound, "linear")


@pytest.mark.parametrize("dt", TYPES, ids=_name)
@pytest.mark.parametrize("m,n,k,kw", [
    (300, 256, 256, {}),
    (4096, 1024, 1024, {}),                       # 2-SM pair tiles (x prefetched into L2)
    (1000, 512, 512, {"tile_n": 64, "pair": 1}),
    (64, 512, 2048, {"splits": 0}),
])
@pytest.mark.parametrize("mode", ["none", "mask_delta", "mask_x"])
def test_linear_residual_half(K, dt, m, n, k, kw, mode):
    g = torch.Generator().manual_seed(m * 3 + n + k + len(mode))
    a = torch.randn(m, k, generator=g).to(dt)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dt)
    b = torch.randn(n, generator=g) * 0.1
    x = (torch.randn(m, n, generator=g) * 3).to(dt)
    valid = torch.rand(m, generator=g) > 0.25
    md, mx = mode == "mask_delta", mode == "mask_x"
    ref, v = om.linear_residual_half(a, w, b, x, valid, md, mx, dt)
    dv = torch.device("cuda:0")
    xg = x.to(dv)
    out = K.linear_residual(a.to(dv), w.to(dv), b.to(dv), xg, None, valid.to(dv), mask_delta=md, mask_x=mx, **kw)
    torch.cuda.synchronize()
    assert out.dtype == dt
    assert torch.equal(xg.cpu(), x)  # x_in untouched when x_out is separate
    _assert_within(out, ref, ULP[dt] * (v.abs() + ref.abs()) + _acc_err(a, w) + 1e-6, "residual")
    if mx:
        assert torch.count_nonzero(out.cpu()[~valid]) == 0
    if md:
        assert torch.equal(out.cpu()[~valid], x[~valid])


@pytest.mark.parametrize("dt", TYPES, ids=_name)
@pytest.mark.parametrize("mode", ["none", "mask_delta", "mask_x"])
def test_linear_residual_ln_half(K, dt, mode):
    """The split-K residual site with its LayerNorm fused into the reduce, in
    a half-precision stream: x_out as the unfused call (bit-identical), normed
    within one ulp of T of the fp32 LayerNorm of x_out."""
    m, n, k = 64, 512, 2048
    g = torch.Generator().manual_seed(n + len(mode))
    a = torch.randn(m, k, generator=g).to(dt)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(dt)
    b = torch.randn(n, generator=g) * 0.1
    x = (torch.randn(m, n, generator=g) * 3).to(dt)
    valid = torch.rand(m, generator=g) > 0.25
    lw = torch.randn(n, generator=g) * 0.1 + 1
    lb = torch.randn(n, generator=g) * 0.1
    md, mx = mode == "mask_delta", mode == "mask_x"
    dv = torch.device("cuda:0")
    args = (a.to(dv), w.to(dv), b.to(dv), x.to(dv))
    x_new, normed = K.linear_residual_ln(*args, None, valid.to(dv), lw.to(dv), lb.to(dv), 1e-5, mask_delta=md,
                                         mask_x=mx, splits=0)
    unfused = K.linear_residual(*args, None, valid.to(dv), mask_delta=md, mask_x=mx, splits=0)
    torch.cuda.synchronize()
    assert x_new.dtype == dt and normed.dtype == dt
    assert torch.equal(x_new, unfused)
    _, yr = om.ln_site_half(x_new.cpu(), None, lw, lb, 1e-5, valid, False, False, False, dt)
    _assert_within(normed, yr, ULP[dt] * yr.abs() + 1e-6, "normed")


@pytest.mark.parametrize("b,h,sq,sk,hd,causal,masked", [
    (2, 4, 256, 256, 64, False, False),
    (1, 2, 300, 300, 64, True, False),
    (2, 2, 200, 333, 128, False, True),
    (1, 4, 1024, 1024, 128, True, False),
])
def test_flash_bf16(K, b, h, sq, sk, hd, causal, masked):
    g = torch.Generator().manual_seed(b * 7 + sq + sk + hd)
    d = h * hd
    q = torch.randn(b, sq, d, generator=g).bfloat16()
    kk = torch.randn(b, sk, d, generator=g).bfloat16()
    vv = torch.randn(b, sk, d, generator=g).bfloat16()
    kv = None
    if masked:
        kv = torch.rand(b, sk, generator=g) > 0.3
        kv[:, 0] = True
    scale = hd ** -0.5

    def heads(t):
        return t.view(t.shape[0], t.shape[1], h, hd).transpose(1, 2)

    ref, lse_ref = om.attention_fp16(heads(q), heads(kk), heads(vv), scale, causal, kv)
    ref = ref.transpose(1, 2).reshape(b, sq, d)
    dv = torch.device("cuda:0")
    out, lse = K.flash_attention(q.to(dv), kk.to(dv), vv.to(dv), h, scale, causal=causal,
                                 key_valid=None if kv is None else kv.to(dv), want_lse=True)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16
    _assert_within(out, ref, 2e-2 * ref.abs() + 4e-3, "attention")
    assert torch.allclose(lse.cpu(), lse_ref, atol=5e-3, rtol=1e-3)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=_name)
@pytest.mark.parametrize("b,h,sq,sk,hd,causal,masked", [
    (2, 4, 256, 256, 64, False, False),
    (1, 2, 300, 300, 64, True, False),
    (2, 2, 200, 333, 128, False, True),
    (1, 4, 1024, 1024, 128, True, False),
])
def test_flash_round_scores(K, dt, b, h, sq, sk, hd, causal, masked):
    """TF_ATTN_ROUND_SCORES: the scores of the eager model in T,
    T(T(q . k) * scale), before the fp32 softmax (oracle
    attention_rounded_scores). q and k hold multiples of 1/8 in [-2, 2], so
    every q . k (a multiple of 1/64 below 512 in magnitude) is exact in fp32
    whatever the summation order, and the kernel and the oracle round the
    same value to T: the scores agree bit for bit. The rounding is exercised
    (fp16 spacing exceeds 1/64 from |q . k| = 32 on; bf16 from 2 on). P is
    rounded to T for the PV product:
    |d| <= 2 ulp(T)*|ref| + 2e-3; the LSE is that of the rounded scores."""
    g = torch.Generator().manual_seed(b * 5 + sq + sk + hd + (1 if dt == torch.bfloat16 else 0))
    d = h * hd
    q = (torch.randint(-16, 17, (b, sq, d), generator=g).float() / 8).to(dt)
    kk = (torch.randint(-16, 17, (b, sk, d), generator=g).float() / 8).to(dt)
    vv = torch.randn(b, sk, d, generator=g).to(dt)
    kv = None
    if masked:
        kv = torch.rand(b, sk, generator=g) > 0.3
        kv[:, 0] = True
    scale = hd ** -0.5

    def heads(t):
        return t.view(t.shape[0], t.shape[1], h, hd).transpose(1, 2)

    ref, lse_ref = om.attention_rounded_scores(heads(q), heads(kk), heads(vv), scale, causal, kv)
    ref = ref.transpose(1, 2).reshape(b, sq, d)
    dv = torch.device("cuda:0")
    out, lse = K.flash_attention(q.to(dv), kk.to(dv), vv.to(dv), h, scale, causal=causal,
                                 key_valid=None if kv is None else kv.to(dv), want_lse=True, round_scores=True)
    torch.cuda.synchronize()
    assert out.dtype == dt
    ulp = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -10
    _assert_within(out, ref, 2 * ulp * ref.abs() + 2e-3, "attention (rounded scores)")
    assert torch.allclose(lse.cpu(), lse_ref, atol=1e-3, rtol=1e-5)
    # fp32 scores (no flag) land measurably further from the rounded-score LSE
    _, lse32 = K.flash_attention(q.to(dv), kk.to(dv), vv.to(dv), h, scale, causal=causal,
                                 key_valid=None if kv is None else kv.to(dv), want_lse=True)
    assert (lse32.cpu() - lse_ref).abs().mean() > 2 * (lse.cpu() - lse_ref).abs().mean()


def test_half_flag_errors(K):
    """Operand types that do not pair are refused, not converted."""
    dv = torch.device("cuda:0")
    a = torch.randn(128, 64, device=dv).half()
    w = torch.randn(64, 64, device=dv).bfloat16()
    b = torch.zeros(64, device=dv)
    with pytest.raises(ValueError):
        K.linear(a, w, b)
    with pytest.raises(ValueError):
        K.linear_residual(a, w.half(), b, torch.zeros(128, 64, device=dv).bfloat16())  # x not in a's type
    from transformer_optimization_b200 import _abi
    with pytest.raises(_abi.TfError):  # bf16 attention takes no FMA-pipe exponentials
        q = torch.randn(1, 128, 64, device=dv).bfloat16()
        K.flash_attention(q, q, q, 1, 0.125, fma_exp_pairs=8)
