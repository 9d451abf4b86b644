"""Kernel-level parity on a B200: each CUDA kernel against the oracle's
statement of the same op (oracle/reference_model.py), on seeded inputs,
through the C ABI (transformer_optimization_b200.kernels -> libtfb200.so).

Tolerances (written per test):
* LayerNorm: fp32 math, different reduction tree -> 2e-5 abs on fp32 output,
  1 fp16 ulp on fp16 output.
* GEMM: fp16 output of an fp32-accumulated sum; the reference value is the
  exact (fp64) sum rounded to fp16, so the kernel may differ by one fp16 ulp
  where the fp32 accumulation order tips a rounding: |d| <= 2e-3*|ref| + 1e-3.
* Attention: P is rounded to fp16 before the PV product (as the reference's
  fp16 SDPA path does): |d| <= 1e-2*|ref| + 3e-3 on fp16 outputs, LSE 2e-3.
"""

import math

import pytest
import torch

from oracle import reference_model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from transformer_optimization_b200 import _abi, kernels
    _abi.load()
    torch.backends.cuda.matmul.allow_tf32 = False
    yield kernels
    assert _abi.device_status() == 0, "a kernel wait ran out"


def _dev():
    return torch.device("cuda:0")


# ----------------------------------------------------------------- LayerNorm
@pytest.mark.parametrize("m,d", [(1, 256), (7, 64), (64, 512), (1000, 1024), (333, 2048), (40, 4096), (5, 136)])
@pytest.mark.parametrize("flags", ["plain", "delta", "mask_delta", "mask_x", "final"])
def test_ln_residual(K, m, d, flags):
    g = torch.Generator().manual_seed(m * 31 + d)
    x = torch.randn(m, d, generator=g) * 2 + 0.5
    delta = (torch.randn(m, d, generator=g) * 0.5).half()
    w = torch.randn(d, generator=g) * 0.1 + 1
    b = torch.randn(d, generator=g) * 0.1
    valid = torch.rand(m, generator=g) > 0.3
    use_delta = flags != "plain"
    md, mx, mo = flags == "mask_delta", flags in ("mask_x", "final"), flags == "final"
    out_f32 = flags == "final"
    xr, yr = om.ln_site(x, delta if use_delta else None, w, b, 1e-5, valid, md, mx, mo)
    dv = _dev()
    xg = x.to(dv)
    x_new, y = K.ln_residual(xg, delta.to(dv) if use_delta else None, w.to(dv), b.to(dv), 1e-5,
                             valid.to(dv), mask_delta=md, mask_x=mx, mask_out=mo, write_x=use_delta,
                             out_dtype=torch.float32 if out_f32 else torch.float16)
    torch.cuda.synchronize()
    if use_delta:
        assert torch.allclose(x_new.cpu(), xr, atol=0, rtol=0)  # same fp32 add
    if out_f32:
        assert torch.allclose(y.cpu(), yr, atol=2e-5, rtol=1e-5)
    else:
        assert torch.allclose(y.float().cpu(), yr.half().float(), atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("d", [256, 1024, 2048])
@pytest.mark.parametrize("flags", ["plain", "delta", "mask_x"])
def test_ln_residual_stream_ring(K, d, flags):
    """Enough rows that every CTA of the streaming LayerNorm cycles its
    shared-memory ring many times (about 12 groups of 8 rows per SM), for the
    two- and three-team configurations (D 2048: two teams and two stages with
    delta, three and three without; D 1024 with delta: two teams, four
    stages; narrower: three teams, six stages)."""
    m = 148 * 8 * 12 + 5
    g = torch.Generator().manual_seed(d + len(flags))
    x = torch.randn(m, d, generator=g) * 2 + 0.5
    delta = (torch.randn(m, d, generator=g) * 0.5).half()
    w = torch.randn(d, generator=g) * 0.1 + 1
    b = torch.randn(d, generator=g) * 0.1
    valid = torch.rand(m, generator=g) > 0.3
    use_delta = flags != "plain"
    mx = flags == "mask_x"
    xr, yr = om.ln_site(x, delta if use_delta else None, w, b, 1e-5, valid, False, mx, False)
    dv = _dev()
    x_new, y = K.ln_residual(x.to(dv), delta.to(dv) if use_delta else None, w.to(dv), b.to(dv), 1e-5, valid.to(dv),
                             mask_x=mx, write_x=use_delta)
    if use_delta:
        assert torch.equal(x_new.cpu(), xr)
    assert torch.allclose(y.float().cpu(), yr.half().float(), atol=2e-3, rtol=1e-3)


def test_ln_residual_in_place(K):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(300, 1024, generator=g)
    delta = torch.randn(300, 1024, generator=g).half()
    w, b = torch.ones(1024), torch.zeros(1024)
    xr, yr = om.ln_site(x, delta, w, b, 1e-5, None, False, False, False)
    xg = x.cuda()
    K.ln_residual(xg, delta.cuda(), w.cuda(), b.cuda(), 1e-5, write_x=True, x_out=xg)
    assert torch.equal(xg.cpu(), xr)


# ----------------------------------------------------------------- GEMM
GEMM_SHAPES = [  # (M, K, N): model projections at small M plus ragged rows
    (256, 256, 768), (256, 256, 1024), (256, 1024, 256), (64, 512, 1536), (64, 2048, 512),
    (300, 1024, 3072), (1000, 1024, 4096), (129, 4096, 1024), (2048, 2048, 6144), (17, 64, 64),
]


def _gemm_inputs(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).half()
    bound = 1 / math.sqrt(k)
    w = (torch.rand(n, k, generator=g) * 2 - 1).mul(bound)
    bias = (torch.rand(n, generator=g) * 2 - 1).mul(bound)
    return a, w, bias


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
@pytest.mark.parametrize("gelu", [False, True])
def test_gemm(K, m, k, n, gelu):
    a, w, bias = _gemm_inputs(m, k, n, m + 7 * k + 13 * n)
    w16 = w.half()
    ref = om.linear_fp16(a, w16, bias, gelu)
    out = K.linear(a.cuda(), w16.cuda(), bias.cuda(), gelu=gelu).float().cpu()
    err = (out - ref).abs()
    assert torch.all(err <= 2e-3 * ref.abs() + 1e-3), f"max err {err.max()}"


def test_gemm_gelu_accuracy(K):
    """GELU epilogue on exactly representable pre-activations: every fp16 value
    in [-12, 12] goes through the GEMM unchanged (one nonzero weight of 1), so
    the output is fp16(gelu(x)) and can be compared with the fp64 GELU value
    by value: within one fp16 unit in the last place plus 1e-6 (the erf
    approximation's absolute error, which shows in the far negative tail where
    GELU is below 1e-4 and fp16 steps are ~1e-7)."""
    xs = torch.arange(-12 * 1024, 12 * 1024 + 1, dtype=torch.float32) / 1024
    xs = torch.unique(xs.half()).float()
    m = xs.numel()
    a = torch.zeros(m, 64, dtype=torch.float16)
    a[:, 0] = xs.half()
    w16 = torch.zeros(128, 64, dtype=torch.float16)
    w16[:, 0] = 1
    bias = torch.zeros(128)
    ref = torch.nn.functional.gelu(xs.double(), approximate="none")
    ref16 = ref.float().half().double()
    out = K.linear(a.cuda(), w16.cuda(), bias.cuda(), gelu=True)[:, 0].double().cpu()
    ulp = (ref16.abs().clamp_min(2.0 ** -14).log2().floor() - 10).exp2()
    diff = (out - ref16).abs()
    assert torch.all(diff <= ulp + 1e-6), f"max diff {diff.max()} at x={xs[diff.argmax()]}"


SPLITK_SHAPES = [(64, 512, 1536), (64, 2048, 512), (256, 1024, 256), (300, 1024, 3072), (17, 4096, 64),
                 (129, 520, 96)]


@pytest.mark.parametrize("m,k,n", SPLITK_SHAPES)
@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("splits", [0, 1, 3, 7])
def test_gemm_splitk(K, m, k, n, gelu, splits):
    """Split-K form (partials in a workspace, fixed-order reduce) against the
    exact sum; the same call twice is bit-identical."""
    a, w, bias = _gemm_inputs(m, k, n, m + 3 * k + n + splits)
    w16 = w.half()
    ref = om.linear_fp16(a, w16, bias, gelu)
    ag, wg, bg = a.cuda(), w16.cuda(), bias.cuda()
    ws = torch.empty(K.splitk_workspace_bytes(m, n, k, splits), dtype=torch.uint8, device="cuda")
    out = K.linear(ag, wg, bg, gelu=gelu, splits=splits, workspace=ws)
    again = K.linear(ag, wg, bg, gelu=gelu, splits=splits, workspace=ws)
    err = (out.float().cpu() - ref).abs()
    assert torch.all(err <= 2e-3 * ref.abs() + 1e-3), f"max err {err.max()}"
    assert torch.equal(out, again)


@pytest.mark.parametrize("mode", ["none", "mask_delta", "mask_x"])
@pytest.mark.parametrize("m,k,n", [(64, 2048, 512), (256, 1024, 256), (1000, 512, 1024)])
def test_gemm_residual_splitk(K, mode, m, k, n):
    a, w, bias = _gemm_inputs(m, k, n, 5 * m + k)
    w16 = w.half()
    g = torch.Generator().manual_seed(m)
    x = torch.randn(m, n, generator=g)
    valid = torch.rand(m, generator=g) > 0.2
    md, mx = mode == "mask_delta", mode == "mask_x"
    ref = om.linear_residual(a, w16, bias, x, valid, md, mx)
    out = K.linear_residual(a.cuda(), w16.cuda(), bias.cuda(), x.cuda(), None, valid.cuda(), mask_delta=md,
                            mask_x=mx, splits=0)
    assert torch.allclose(out.cpu(), ref, atol=1e-4, rtol=1e-5)


@pytest.mark.parametrize("mode", ["none", "mask_delta", "mask_x", "final"])
@pytest.mark.parametrize("m,k,n", [(64, 2048, 512), (256, 1024, 256), (200, 512, 1024), (37, 256, 4096)])
def test_gemm_residual_ln_splitk(K, mode, m, k, n):
    """Split-K residual projection whose reduce kernel also runs the
    LayerNorm of the result: x_out bit-identical to the unfused split-K call,
    normed against the oracle's LayerNorm of it (1 fp16 ulp; fp32 output
    2e-5), masked rows of the final form zero."""
    a, w, bias = _gemm_inputs(m, k, n, 7 * m + k + n)
    w16 = w.half()
    g = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, n, generator=g)
    valid = torch.rand(m, generator=g) > 0.2
    lw = torch.randn(n, generator=g) * 0.1 + 1
    lb = torch.randn(n, generator=g) * 0.1
    md, mx, mo = mode == "mask_delta", mode in ("mask_x", "final"), mode == "final"
    out_dtype = torch.float32 if mode == "final" else torch.float16
    dv = torch.device("cuda")
    ag, wg, bg, xg, vg = a.to(dv), w16.to(dv), bias.to(dv), x.to(dv), valid.to(dv)
    x_new, normed = K.linear_residual_ln(ag, wg, bg, xg, None, vg, lw.to(dv), lb.to(dv), 1e-5, mask_delta=md,
                                         mask_x=mx, mask_out=mo, out_dtype=out_dtype, splits=0)
    unfused = K.linear_residual(ag, wg, bg, xg, None, vg, mask_delta=md, mask_x=mx, splits=0)
    torch.cuda.synchronize()
    assert torch.equal(x_new, unfused)
    ref_x = om.linear_residual(a, w16, bias, x, valid, md, mx)
    assert torch.allclose(x_new.cpu(), ref_x, atol=1e-4, rtol=1e-5)
    _, yr = om.ln_site(x_new.cpu(), None, lw, lb, 1e-5, valid, False, False, mo)
    if out_dtype == torch.float32:
        assert torch.allclose(normed.cpu(), yr, atol=2e-5, rtol=1e-5)
        assert torch.count_nonzero(normed.cpu()[~valid]) == 0
    else:
        assert torch.allclose(normed.float().cpu(), yr.half().float(), atol=2e-3, rtol=1e-3)


def test_gemm_splitk_workspace_checks(K):
    from transformer_optimization_b200 import _abi
    a, w, bias = _gemm_inputs(64, 1024, 256, 1)
    need = K.splitk_workspace_bytes(64, 256, 1024, 4)
    assert need == 4 * 64 * 256 * 4
    small = torch.empty(need - 16, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        K.linear(a.cuda(), w.half().cuda(), bias.cuda(), splits=4, workspace=small)
    with pytest.raises(_abi.TfError):  # the library's own check
        _abi.call("tf_gemm_splitk", a.cuda().data_ptr(), 1024, w.half().cuda().data_ptr(), 1024,
                  bias.cuda().data_ptr(), torch.empty(64, 256, dtype=torch.float16, device="cuda").data_ptr(), 256,
                  64, 256, 1024, 0, 4, small.data_ptr(), small.numel(), 0)


@pytest.mark.parametrize("tile_n", [64, 128, 256])
def test_gemm_tiles(K, tile_n):
    m, k, n = 777, 1024, 1536
    a, w, bias = _gemm_inputs(m, k, n, tile_n)
    w16 = w.half()
    ref = om.linear_fp16(a, w16, bias, False)
    out = K.linear(a.cuda(), w16.cuda(), bias.cuda(), tile_n=tile_n).float().cpu()
    assert torch.all((out - ref).abs() <= 2e-3 * ref.abs() + 1e-3)


@pytest.mark.parametrize("m", [64, 300, 1000, 4096])
@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("gelu", [False, True])
def test_gemm_pair_tiles(K, m, tile_n, gelu):
    """2-SM (CTA pair, cta_group::2) tiles, including row tails that leave
    the second CTA of a pair partly or fully outside M."""
    k, n = 1024, 1536
    a, w, bias = _gemm_inputs(m, k, n, m + tile_n)
    w16 = w.half()
    ref = om.linear_fp16(a, w16, bias, gelu)
    out = K.linear(a.cuda(), w16.cuda(), bias.cuda(), gelu=gelu, tile_n=tile_n, pair=2).float().cpu()
    err = (out - ref).abs()
    assert torch.all(err <= 2e-3 * ref.abs() + 1e-3), f"max err {err.max()}"


@pytest.mark.parametrize("k", [64, 320, 960])
@pytest.mark.parametrize("pair", [1, 2])
def test_gemm_odd_kblock_groups(K, k, pair):
    """The main loop consumes stages in groups of two 64-wide k-blocks; an odd
    count (1, 5, 15 blocks) ends with a group of one, on both kernel forms."""
    m, n = 1000, 1536
    a, w, bias = _gemm_inputs(m, k, n, k + pair)
    w16 = w.half()
    ref = om.linear_fp16(a, w16, bias, False)
    out = K.linear(a.cuda(), w16.cuda(), bias.cuda(), tile_n=256 if pair == 2 else 128, pair=pair).float().cpu()
    err = (out - ref).abs()
    assert torch.all(err <= 2e-3 * ref.abs() + 1e-3), f"max err {err.max()}"


@pytest.mark.parametrize("mode", ["none", "mask_delta", "mask_x"])
def test_gemm_residual_large(K, mode):
    """Large enough for the automatic choice to take 2-SM tiles."""
    m, k, n = 9000, 512, 1024
    a, w, bias = _gemm_inputs(m, k, n, 77)
    w16 = w.half()
    g = torch.Generator().manual_seed(2)
    x = torch.randn(m, n, generator=g)
    valid = torch.rand(m, generator=g) > 0.1
    md, mx = mode == "mask_delta", mode == "mask_x"
    ref = om.linear_residual(a, w16, bias, x, valid, md, mx)
    out = K.linear_residual(a.cuda(), w16.cuda(), bias.cuda(), x.cuda(), None, valid.cuda(), mask_delta=md,
                            mask_x=mx)
    assert torch.allclose(out.cpu(), ref, atol=1e-4, rtol=1e-5)


def test_gemm_strided_output(K):
    """QKV-style: write into a column slice of a wider buffer."""
    m, k, n = 200, 512, 512
    a, w, bias = _gemm_inputs(m, k, n, 9)
    w16 = w.half()
    big = torch.zeros(m, 3 * n, dtype=torch.float16, device="cuda")
    K.linear(a.cuda(), w16.cuda(), bias.cuda(), out=big[:, n:2 * n])
    ref = om.linear_fp16(a, w16, bias, False)
    assert torch.all(((big[:, n:2 * n].float().cpu()) - ref).abs() <= 2e-3 * ref.abs() + 1e-3)
    assert torch.count_nonzero(big[:, :n]) == 0 and torch.count_nonzero(big[:, 2 * n:]) == 0


@pytest.mark.parametrize("m,k,n", [(300, 1024, 1024), (64, 2048, 512), (1000, 4096, 2048), (129, 200, 256)])
@pytest.mark.parametrize("mode", ["none", "mask_delta", "mask_x"])
def test_gemm_residual(K, m, k, n, mode):
    """fp32 residual epilogue: x_out = mask_x(x_in + mask_delta(a @ w.T + b)).
    The delta is an fp32-accumulated sum of fp16 products: |d| <= 1e-4 + 1e-5|x|."""
    a, w, bias = _gemm_inputs(m, k, n, m + k + n)
    w16 = w.half()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(m, n, generator=g) * 3
    valid = torch.rand(m, generator=g) > 0.25
    md, mx = mode == "mask_delta", mode == "mask_x"
    ref = om.linear_residual(a, w16, bias, x, valid, md, mx)
    xg = x.cuda()
    out = K.linear_residual(a.cuda(), w16.cuda(), bias.cuda(), xg, None, valid.cuda(), mask_delta=md, mask_x=mx)
    assert torch.equal(xg.cpu(), x)  # x_in untouched when x_out is separate
    assert torch.allclose(out.cpu(), ref, atol=1e-4, rtol=1e-5)
    # in place
    K.linear_residual(a.cuda(), w16.cuda(), bias.cuda(), xg, xg, valid.cuda(), mask_delta=md, mask_x=mx)
    assert torch.allclose(xg.cpu(), ref, atol=1e-4, rtol=1e-5)
    if mx:
        assert torch.count_nonzero(xg.cpu()[~valid]) == 0
    if md:
        assert torch.equal(xg.cpu()[~valid], x[~valid])


@pytest.mark.parametrize("k", [1024, 8192, 200])
def test_gemm_split_weight(K, k):
    """[W_hi | W_lo] weights reproduce the fp32 weight: the error against the
    fp32-weight product is far below the plain fp16-weight error."""
    m, n = 256, 512
    a, w, bias = _gemm_inputs(m, k, n, k)
    x = torch.zeros(m, n)
    ref = om.linear_residual(a, w, bias, x, None, False, False)  # fp32 weight
    plain = K.linear_residual(a.cuda(), w.half().cuda(), bias.cuda(), x.cuda()).cpu()
    split = K.linear_residual(a.cuda(), K.split_weight(w).cuda(), bias.cuda(), x.cuda(), w_split=True).cpu()
    e_plain = (plain - ref).abs().max().item()
    e_split = (split - ref).abs().max().item()
    # what is left is the fp32 accumulation over K products
    assert e_split < e_plain / 4, (e_split, e_plain)
    assert torch.allclose(split, ref, atol=1e-4 * math.sqrt(k / 1024), rtol=1e-5)
    # the fp16-output GEMM takes split weights too
    out16 = K.linear(a.cuda(), K.split_weight(w).cuda(), bias.cuda(), w_split=True).float().cpu()
    r16 = ref.half().float()
    assert torch.all((out16 - r16).abs() <= 2e-3 * r16.abs() + 1e-3)


# ----------------------------------------------------------------- attention
ATTN_CASES = [  # (B, H, Sq, Sk, hd, causal, masked)
    (2, 4, 128, 128, 64, False, False),
    (2, 4, 128, 128, 64, True, False),
    (1, 8, 64, 64, 64, False, False),
    (1, 2, 300, 300, 128, False, False),
    (1, 2, 300, 300, 128, True, False),
    (3, 2, 200, 200, 64, False, True),
    (2, 3, 257, 257, 64, True, True),
    (1, 2, 1000, 1000, 128, True, False),
    (2, 16, 512, 512, 64, False, False),
]


def _qkv(b, h, s, hd, seed):
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(b, s, 3 * h * hd, generator=g) * 1.5).half()
    return qkv


@pytest.mark.parametrize("b,h,sq,sk,hd,causal,masked", ATTN_CASES)
@pytest.mark.parametrize("exp_f16x2", [False, True])
def test_flash_packed_qkv(K, b, h, sq, sk, hd, causal, masked, exp_f16x2):
    d = h * hd
    qkv = _qkv(b, h, sq, hd, sq + hd)
    kv_valid = None
    if masked:
        kv_valid = torch.arange(sk)[None, :] < torch.randint(1, sk + 1, (b,), generator=torch.Generator().manual_seed(1))[:, None]
    q = qkv[..., :d].reshape(b, sq, h, hd).transpose(1, 2)
    k = qkv[..., d:2 * d].reshape(b, sk, h, hd).transpose(1, 2)
    v = qkv[..., 2 * d:].reshape(b, sk, h, hd).transpose(1, 2)
    ref, lse_ref = om.attention_fp16(q, k, v, hd ** -0.5, causal, kv_valid)
    ref = ref.transpose(1, 2).reshape(b, sq, d)
    g = qkv.cuda()
    out, lse = K.flash_attention(g[..., :d], g[..., d:2 * d], g[..., 2 * d:], h, hd ** -0.5, causal=causal,
                                 key_valid=None if kv_valid is None else kv_valid.cuda(), want_lse=True,
                                 exp_f16x2=exp_f16x2)
    out = out.float().cpu()
    err = (out - ref).abs()
    assert torch.all(err <= 1e-2 * ref.abs() + 3e-3), f"max err {err.max()}"
    lse = lse.cpu()
    fin = torch.isfinite(lse_ref)
    assert torch.equal(fin, torch.isfinite(lse))
    assert torch.allclose(lse[fin], lse_ref[fin], atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("pairs,f16x2", [(8, False), (16, False), (24, False), (16, True)])
@pytest.mark.parametrize("b,h,sq,hd,causal,masked", [(2, 4, 300, 64, True, True), (1, 2, 513, 128, False, False)])
def test_flash_fma_exp(K, pairs, f16x2, b, h, sq, hd, causal, masked):
    """Part of the exponentials on the FMA pipes (fp32 or binary16 built from
    a polynomial) gives the same attention within the fp16-P tolerance."""
    d = h * hd
    qkv = _qkv(b, h, sq, hd, pairs + sq)
    kv_valid = None
    if masked:
        kv_valid = torch.arange(sq)[None, :] < torch.tensor([sq - 37 * (i + 1) for i in range(b)])[:, None]
    split = lambda t: t.reshape(b, sq, h, hd).transpose(1, 2)
    ref, lse_ref = om.attention_fp16(split(qkv[..., :d]), split(qkv[..., d:2 * d]), split(qkv[..., 2 * d:]),
                                     hd ** -0.5, causal, kv_valid)
    ref = ref.transpose(1, 2).reshape(b, sq, d)
    g = qkv.cuda()
    out, lse = K.flash_attention(g[..., :d], g[..., d:2 * d], g[..., 2 * d:], h, hd ** -0.5, causal=causal,
                                 key_valid=None if kv_valid is None else kv_valid.cuda(), want_lse=True,
                                 fma_exp_pairs=pairs, exp_f16x2=f16x2)
    out = out.float().cpu()
    assert torch.all((out - ref).abs() <= 1e-2 * ref.abs() + 3e-3), (out - ref).abs().max()
    fin = torch.isfinite(lse_ref)
    assert torch.allclose(lse.cpu()[fin], lse_ref[fin], atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("hd", [64, 128])
def test_flash_offsets_and_f32_out(K, hd):
    """Context-parallel block: queries at global positions [q0, q0+Sq), keys
    at [k0, k0+Sk); causal mask on global positions; fp32 output."""
    b, h, sq, sk = 1, 2, 200, 300
    q0, k0 = 500, 380
    g = torch.Generator().manual_seed(hd)
    q = (torch.randn(b, sq, h * hd, generator=g)).half()
    kk = (torch.randn(b, sk, h * hd, generator=g)).half()
    vv = (torch.randn(b, sk, h * hd, generator=g)).half()
    split = lambda t, s: t.reshape(b, s, h, hd).transpose(1, 2)
    ref, lse_ref = om.attention_fp16(split(q, sq), split(kk, sk), split(vv, sk), hd ** -0.5, True, None,
                                     q_offset=q0 - k0)
    ref = ref.transpose(1, 2).reshape(b, sq, h * hd)
    out, lse = K.flash_attention(q.cuda(), kk.cuda(), vv.cuda(), h, hd ** -0.5, causal=True, q_pos0=q0,
                                 k_pos0=k0, out_dtype=torch.float32, want_lse=True)
    out = out.cpu()
    assert torch.all((out - ref).abs() <= 1e-2 * ref.abs() + 3e-3)
    fin = torch.isfinite(lse_ref)
    assert torch.equal(fin, torch.isfinite(lse.cpu()))
    assert torch.allclose(lse.cpu()[fin], lse_ref[fin], atol=2e-3)


def test_flash_fully_masked_rows(K):
    """Queries before every key (causal) get out = 0 and lse = -inf."""
    b, h, hd, sq, sk = 1, 1, 64, 130, 128
    q = torch.randn(b, sq, hd).half().cuda()
    k = torch.randn(b, sk, hd).half().cuda()
    out, lse = K.flash_attention(q, k, k, h, 0.125, causal=True, q_pos0=0, k_pos0=1000, want_lse=True)
    assert torch.count_nonzero(out) == 0
    assert torch.all(torch.isneginf(lse))


@pytest.mark.parametrize("b,s,h,hd", [(2, 100, 4, 64), (1, 300, 16, 64), (2, 77, 8, 128), (1, 50, 40, 32)])
def test_attn_merge(K, b, s, h, hd):
    """Row-per-warp form (heads <= 32) and the per-head form (40 heads)."""
    g = torch.Generator().manual_seed(3)
    oa = torch.randn(b, s, h * hd, generator=g)
    ob = torch.randn(b, s, h * hd, generator=g)
    la = torch.randn(b, h, s, generator=g)
    lb = torch.randn(b, h, s, generator=g)
    la[0, 0, :5] = -math.inf
    L = torch.logaddexp(la, lb)
    wa = torch.exp(la - L).transpose(1, 2).repeat_interleave(hd, dim=2)
    wb = torch.exp(lb - L).transpose(1, 2).repeat_interleave(hd, dim=2)
    ref = oa * wa + ob * wb
    oag, lag = oa.cuda(), la.cuda()
    o16 = torch.empty(b, s, h * hd, dtype=torch.float16, device="cuda")
    K.attn_merge(oag, lag, ob.cuda(), lb.cuda(), h, out16=o16)
    assert torch.allclose(oag.cpu(), ref, atol=1e-5, rtol=1e-5)
    assert torch.allclose(lag.cpu(), L, atol=1e-5)
    assert torch.allclose(o16.float().cpu(), ref, atol=2e-3, rtol=1e-3)
