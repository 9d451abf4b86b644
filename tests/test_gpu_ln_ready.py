"""The overlapped residual GEMM -> LayerNorm pair (tf_gemm_residual_ready +
tf_ln_ready) on a B200.

The LayerNorm starts while the GEMM's last wave still runs and reads each
8-row group once the GEMM's epilogue has counted all D columns of it. The
pair must give exactly what the same GEMM followed by the stand-alone
LayerNorm gives (same per-row arithmetic: bit-identical), which is checked
against the oracle's LayerNorm site, and must leave every counter at zero.
A chain of in-place steps makes an early read visible: a row read before the
GEMM stored it would still hold the previous step's values.

The count wait fails without a fault: a count above its target is refused at
once, and a count that nothing completes runs out after the 2 s wait bound;
both record device code 107 and leave the device usable.
"""

import pytest
import torch

from oracle import reference_model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K():
    from transformer_optimization_b200 import _abi, kernels
    _abi.load()
    yield kernels
    assert _abi.device_status() == 0, "a kernel wait ran out"


def _inputs(m, k, n, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * 0.5).to(torch.float16 if dtype == torch.float32 else dtype)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(a.dtype)
    bias = torch.randn(n, generator=g) * 0.1
    x = (torch.randn(m, n, generator=g) * 2 + 0.3).to(dtype)
    valid = torch.rand(m, generator=g) > 0.25
    lnw = torch.randn(n, generator=g) * 0.1 + 1
    lnb = torch.randn(n, generator=g) * 0.1
    return a, w, bias, x, valid, lnw, lnb


CASES = [
    # m, k, n, residual dtype, mask mode, final LayerNorm (mask_out, fp32 out)
    (16384, 1024, 1024, torch.float32, "none", False),      # c3: 2-SM 256-wide tiles
    (9000, 512, 1024, torch.float32, "mask_delta", False),
    (1000, 4096, 1024, torch.float32, "mask_x", True),
    (300, 1024, 768, torch.float32, "none", False),         # one-CTA tiles, N not a multiple of 256
    (4099, 1024, 2048, torch.float32, "mask_x", False),     # ragged last group, D = 2048
    (2048, 1024, 1024, torch.float16, "none", False),       # half-precision models: x in T
    (2048, 1024, 1024, torch.bfloat16, "mask_x", True),
]


@pytest.mark.parametrize("m,k,n,dtype,mode,final", CASES)
def test_ready_pair_matches_sequential(K, m, k, n, dtype, mode, final):
    a, w, bias, x, valid, lnw, lnb = _inputs(m, k, n, dtype, m + n)
    dv = torch.device("cuda:0")
    a, w, bias, x, valid, lnw, lnb = (t.to(dv) for t in (a, w, bias, x, valid, lnw, lnb))
    md, mx = mode == "mask_delta", mode == "mask_x"
    out_dtype = torch.float32 if final else None
    ready = K.ready_counters(m, dv)
    xr = K.linear_residual(a, w, bias, x, None, valid, mask_delta=md, mask_x=mx, ready=ready)
    yr = K.ln_ready(xr, lnw, lnb, 1e-5, ready, valid, mask_out=final, out_dtype=out_dtype)
    xs = K.linear_residual(a, w, bias, x, None, valid, mask_delta=md, mask_x=mx)
    _, ys = K.ln_residual(xs, None, lnw, lnb, 1e-5, valid, mask_out=final, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert torch.equal(xr, xs)
    assert torch.equal(yr, ys)
    assert int(ready.abs().sum()) == 0, "counters not consumed"
    if dtype == torch.float32:
        _, y_ref = om.ln_site(xs.cpu(), None, lnw.cpu(), lnb.cpu(), 1e-5, valid.cpu(), False, False, final)
        if final:
            assert torch.allclose(yr.cpu(), y_ref, atol=2e-5, rtol=1e-5)
        else:
            assert torch.allclose(yr.float().cpu(), y_ref.half().float(), atol=2e-3, rtol=1e-3)


def test_ready_pair_chain_in_place(K):
    """Ten in-place residual steps, each followed by its LayerNorm, on one set
    of counters: every normed output equals the sequential path's."""
    m, k, n = 16384, 1024, 1024
    a, w, bias, x, valid, lnw, lnb = (t.cuda() for t in _inputs(m, k, n, torch.float32, 5))
    ready = K.ready_counters(m, x.device)
    xa, xb = x.clone(), x.clone()
    outs_a, outs_b = [], []
    for step in range(10):
        K.linear_residual(a, w, bias, xa, xa, ready=ready)
        outs_a.append(K.ln_ready(xa, lnw, lnb, 1e-5, ready))
        K.linear_residual(a, w, bias, xb, xb)
        outs_b.append(K.ln_residual(xb, None, lnw, lnb, 1e-5)[1])
    torch.cuda.synchronize()
    assert torch.equal(xa, xb)
    for step, (ya, yb) in enumerate(zip(outs_a, outs_b)):
        assert torch.equal(ya, yb), f"step {step} differs"
    assert int(ready.abs().sum()) == 0


def test_ready_count_above_target_is_refused(K):
    from transformer_optimization_b200 import _abi
    m, n = 256, 1024
    x = torch.randn(m, n, device="cuda")
    lnw, lnb = torch.ones(n, device="cuda"), torch.zeros(n, device="cuda")
    ready = K.ready_counters(m, x.device)
    ready[:(m + 7) // 8] = n + 32  # group counts above the row width; ticket counters zero
    K.ln_ready(x, lnw, lnb, 1e-5, ready)
    assert _abi.device_status() == 107
    # the device stays usable
    ready.zero_()
    xs = K.linear_residual(torch.randn(m, 64, device="cuda").half(), torch.randn(n, 64, device="cuda").half(),
                           torch.zeros(n, device="cuda"), x, None, ready=ready)
    y = K.ln_ready(xs, lnw, lnb, 1e-5, ready)
    torch.cuda.synchronize()
    assert torch.equal(y, K.ln_residual(xs, None, lnw, lnb, 1e-5)[1])
    assert _abi.device_status() == 0


def test_ready_count_never_completed_times_out(K):
    """Counters that no GEMM fills: the LayerNorm's count wait runs out after
    its 2 s bound, records 107, and the kernel returns."""
    from transformer_optimization_b200 import _abi
    m, n = 64, 256
    x = torch.randn(m, n, device="cuda")
    lnw, lnb = torch.ones(n, device="cuda"), torch.zeros(n, device="cuda")
    ready = K.ready_counters(m, x.device)
    K.ln_ready(x, lnw, lnb, 1e-5, ready)
    assert _abi.device_status() == 107
    y = K.ln_residual(x, None, lnw, lnb, 1e-5)[1]
    torch.cuda.synchronize()
    assert torch.isfinite(y.float()).all()
    assert _abi.device_status() == 0


def test_ready_argument_checks(K):
    x = torch.randn(64, 256, device="cuda")
    lnw, lnb = torch.ones(256, device="cuda"), torch.zeros(256, device="cuda")
    with pytest.raises(ValueError):
        K.ln_ready(x, lnw, lnb, 1e-5, torch.zeros(7, dtype=torch.int32, device="cuda"))  # too few groups
    with pytest.raises(ValueError):
        K.ln_ready(x, lnw, lnb, 1e-5, torch.zeros(8, dtype=torch.int64, device="cuda"))
    a, w = torch.randn(64, 64, device="cuda").half(), torch.randn(256, 64, device="cuda").half()
    with pytest.raises(ValueError):
        K.linear_residual(a, w, lnb, x, None, ready=K.ready_counters(64, x.device), splits=0)
    wide = torch.randn(8, 4096, device="cuda")
    from transformer_optimization_b200._abi import TfError
    with pytest.raises(TfError):
        K.ln_ready(wide, torch.ones(4096, device="cuda"), torch.zeros(4096, device="cuda"), 1e-5,
                   K.ready_counters(8, wide.device))
