"""Pin the oracle against the real reference's outputs (CPU, no GPU).

`tests/golden/golden_cases.pt` was produced by `tests/golden/make_golden.py`,
which runs the reference's own `BaselineTransformer` /
`QueryTiledBaselineTransformer` (torch_transformer_benchmark.py:135-248,
341-437). These tests rebuild each case with the oracle only and require:

* the same weights and inputs (state_dict and x checksums),
* the same outputs: bit-equal when this host runs the torch build that made
  the fixtures, within 1e-5 otherwise (a different BLAS may reorder fp32 sums).
"""

from pathlib import Path

import pytest
import torch

from oracle import reference_model as om
from transformer_optimization_b200.config import TransformerConfig

GOLDEN = torch.load(Path(__file__).parent / "golden" / "golden_cases.pt", weights_only=False)


def _sd_checksum(p):
    tot = torch.zeros((), dtype=torch.float64)
    wsum = torch.zeros((), dtype=torch.float64)
    for i, (k, v) in enumerate(p.items()):
        v = v.double()
        tot += v.sum()
        wsum += (v.flatten()[:: max(1, v.numel() // 97)] * (i + 1)).sum()
    return torch.stack([tot, wsum])


@pytest.mark.parametrize("name", sorted(GOLDEN["cases"]))
def test_oracle_matches_reference(name):
    rec = GOLDEN["cases"][name]
    b, s, d, h, f, l, causal, pad, qtile, seed = rec["shape"]
    cfg = TransformerConfig(b, s, d, h, f, l, causal)
    torch.set_num_threads(min(8, torch.get_num_threads()))
    p, x = om.seeded_case(cfg, seed)
    assert torch.allclose(_sd_checksum(p), rec["sd_checksum"], rtol=0, atol=1e-9), \
        "oracle init_params does not rebuild the reference's weights"
    mask = rec["mask"]
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
        assert torch.equal(om.padded_mask(cfg, pad, seed + 1000), mask)
    assert torch.allclose(torch.stack([x.double().sum(), (x.double() ** 2).sum()]),
                          rec["x_checksum"], rtol=0, atol=1e-9)
    with torch.inference_mode():
        y = om.forward(p, cfg, x, mask, query_tile=qtile, ffn_row_chunk=4096 if qtile else None)
    if rec["y_index"] is not None:
        y = y[:, rec["y_index"], :]
    tol = 0.0 if GOLDEN["torch_version"] == torch.__version__ else 1e-5
    assert torch.allclose(y, rec["y"], rtol=0, atol=tol), (y - rec["y"]).abs().max()


GOLDEN_HALF = torch.load(Path(__file__).parent / "golden" / "golden_half_cases.pt", weights_only=False)


@pytest.mark.parametrize("name", sorted(GOLDEN_HALF["cases"]))
def test_oracle_half_matches_reference(name):
    """The oracle's forward on fp16 / bf16 parameters and input reproduces the
    reference's eager model converted with .to(dtype): bit-equal on the torch
    build that made the fixture, within a few ulps of the type otherwise."""
    rec = GOLDEN_HALF["cases"][name]
    b, s, d, h, f, l, causal, pad, seed = rec["shape"]
    dt = rec["dtype"]
    cfg = TransformerConfig(b, s, d, h, f, l, causal)
    torch.set_num_threads(min(8, torch.get_num_threads()))
    p, x = om.seeded_case(cfg, seed)
    assert torch.allclose(_sd_checksum(p), rec["sd_checksum"], rtol=0, atol=1e-9)
    mask = rec["mask"]
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    with torch.inference_mode():
        y = om.forward({k: v.to(dt) for k, v in p.items()}, cfg, x.to(dt), mask)
    assert y.dtype == dt
    if rec["y_index"] is not None:
        y = y[:, rec["y_index"], :]
    if GOLDEN_HALF["torch_version"] == torch.__version__:
        assert torch.equal(y, rec["y"])
    else:
        ulp = 2.0 ** -10 if dt == torch.float16 else 2.0 ** -7
        assert torch.allclose(y.float(), rec["y"].float(), rtol=4 * ulp, atol=4 * ulp)


GOLDEN_INPUTS = torch.load(Path(__file__).parent / "golden" / "golden_harness_inputs.pt", weights_only=False)


@pytest.mark.parametrize("name", sorted(GOLDEN_INPUTS["cases"]))
def test_harness_case_matches_reference(name):
    """oracle.harness_case draws the harness's per-trial input and mask
    (generate_random_case, torch_transformer_benchmark.py:4359-4397): same x
    (checksums and first elements) and mask on the CPU."""
    rec = GOLDEN_INPUTS["cases"][name]
    b, s, d, h, f, l, seed, pad, scale = rec["args"]
    cfg = TransformerConfig(b, s, d, h, f, l, False)
    x, mask = om.harness_case(cfg, torch.device("cpu"), torch.float32, seed, pad, scale)
    assert torch.equal(mask, rec["mask"])
    assert torch.equal(x.flatten()[:64], rec["x_head"])
    xd = x.double().flatten()
    w = torch.arange(1, xd.numel() + 1, dtype=torch.float64) % 97
    assert torch.allclose(torch.stack([xd.sum(), (xd * xd).sum(), (xd * w).sum()]), rec["x_checksum"],
                          rtol=1e-12, atol=1e-9)


def test_compare_outputs_or_criterion():
    """compare_outputs uses (abs<=atol) OR (abs<=rtol*|ref|), not isclose."""
    ref = torch.tensor([1.0, 0.1, 0.0, float("nan")])
    # 0.02 abs on 1.0 passes by rtol, 0.0021 abs on 0.1 fails both,
    # 0.0019 on 0 passes by atol, NaN always fails.
    opt = torch.tensor([1.02, 0.1021, 0.0019, 0.0])
    r = om.compare_outputs(ref, opt, rtol=0.02, atol=0.002)
    assert not r.passed
    assert r.failed_elements == 2
    r2 = om.compare_outputs(ref[:3], opt[:3].clone().index_fill_(0, torch.tensor([1]), 0.1019))
    assert r2.passed


def test_query_tiled_equals_dense():
    cfg = TransformerConfig(1, 70, 64, 2, 96, 1, True)
    p, x = om.seeded_case(cfg, 11)
    y0 = om.forward(p, cfg, x)
    y1 = om.forward(p, cfg, x, query_tile=16, ffn_row_chunk=33)
    assert torch.allclose(y0, y1, atol=1e-5)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
def test_half_helpers_match_eager_ops(dt):
    """The oracle's per-kernel statements for half-precision models
    (linear_half, linear_residual_half, ln_site_half) agree with the eager ops
    the reference's model runs in that type (nn.Linear, F.gelu, the residual
    add, nn.LayerNorm on T tensors, torch_transformer_benchmark.py:162-248) on
    the CPU: within two ulps of T (ATen accumulates in fp32, the oracle
    exactly)."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(5)
    ulp = 2.0 ** -10 if dt == torch.float16 else 2.0 ** -7
    a = torch.randn(48, 96, generator=g).to(dt)
    w = (torch.randn(64, 96, generator=g) * 96 ** -0.5).to(dt)
    b = (torch.randn(64, generator=g) * 0.1).to(dt)
    x = (torch.randn(48, 64, generator=g) * 2).to(dt)
    lw = (torch.randn(64, generator=g) * 0.1 + 1).to(dt)
    lb = (torch.randn(64, generator=g) * 0.1).to(dt)

    def close(got, want):
        want = want.float()
        assert torch.all((got.float() - want).abs() <= 2 * ulp * want.abs() + 1e-6)

    h = F.linear(a, w, b)
    close(om.linear_half(a, w, b.float(), False, dt), h)
    close(om.linear_half(a, w, b.float(), True, dt), F.gelu(h, approximate="none"))
    x_new, _ = om.linear_residual_half(a, w, b.float(), x, None, False, False, dt)
    close(x_new, x + h)
    delta = (torch.randn(48, 64, generator=g) * 0.5).to(dt)
    xs, y = om.ln_site_half(x, delta, lw.float(), lb.float(), 1e-5, None, False, False, False, dt)
    assert torch.equal(xs, (x + delta).float())
    close(y.to(dt), F.layer_norm(x + delta, (64,), lw, lb, 1e-5))
