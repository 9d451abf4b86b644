"""End-to-end parity on a B200: UserOptimizedTransformer (sm_100a kernels via
the C ABI) against the oracle's fp32 eager model on identical seeded weights
and inputs, judged by the reference's own gate (compare_outputs,
torch_transformer_benchmark.py:4548-4615): |d| <= 0.002 OR |d| <= 0.02*|ref|
with ZERO failing elements.

Small configs run the oracle on the CPU. c3-c5 run the same oracle code on
the GPU in strict fp32 (TF32 off); c4/c5 use its query-tiled attention and
row-chunked FFN (the reference's QueryTiledBaselineTransformer arithmetic)
to bound memory.
"""

import pytest
import torch

from oracle import reference_model as om
from transformer_optimization_b200 import NAMED_CONFIGS, TransformerConfig, UserOptimizedTransformer
from transformer_optimization_b200._abi import TfError

pytestmark = pytest.mark.gpu
ATOL, RTOL = 0.002, 0.02


def _build(cfg, seed=0):
    p, x = om.seeded_case(cfg, seed)
    model = UserOptimizedTransformer(cfg)
    model.load_state_dict(p, strict=True)
    return p, x, model.cuda().eval()


def _check(ref, out):
    r = om.compare_outputs(ref.float().cpu(), out.float().cpu(), rtol=RTOL, atol=ATOL)
    assert r.passed, (f"{r.failed_elements}/{r.total_elements} failed, max_abs={r.max_abs_error:.3g} "
                      f"at {r.worst_index} ref={r.reference_at_worst:.6g} opt={r.optimized_at_worst:.6g}")
    return r


SMALL = {
    "c1": NAMED_CONFIGS["c1"],
    "c1_causal": TransformerConfig(2, 128, 256, 4, 1024, 2, True),
    "c2": NAMED_CONFIGS["c2"],
    "c2_causal": TransformerConfig(1, 64, 512, 8, 2048, 6, True),
    "ragged_hd128": TransformerConfig(1, 100, 256, 2, 512, 1, False),
    "ragged_causal": TransformerConfig(3, 300, 128, 2, 256, 2, True),
    "d2048_hd128": TransformerConfig(2, 256, 2048, 16, 8192, 2, False),
}


@pytest.mark.parametrize("name", sorted(SMALL))
def test_small_configs(name):
    cfg = SMALL[name]
    p, x, model = _build(cfg)
    ref = om.forward(p, cfg, x)
    with torch.inference_mode():
        out = model(x.cuda())
    _check(ref, out)


@pytest.mark.parametrize("causal", [False, True])
def test_partial_mask(causal):
    cfg = TransformerConfig(3, 200, 256, 4, 1024, 2, causal)
    p, x, model = _build(cfg, seed=7)
    mask = om.padded_mask(cfg, 0.4, 1007)
    x = x.masked_fill(~mask[..., None], 0)
    ref = om.forward(p, cfg, x, mask)
    with torch.inference_mode():
        out = model(x.cuda(), mask.cuda())
    _check(ref, out)
    assert torch.count_nonzero(out.cpu()[~mask]) == 0


def test_all_true_mask_and_graph_replay():
    """The harness always passes an all-True mask (torch_transformer_benchmark.py:
    4380-4384). Replays are bit-identical, the input is not mutated and the
    output does not alias the graph's static buffer."""
    cfg = NAMED_CONFIGS["c2"]
    p, x, model = _build(cfg)
    xg = x.cuda()
    x_copy = xg.clone()
    mask = torch.ones(1, 64, dtype=torch.bool, device="cuda")
    with torch.inference_mode():
        a = model(xg, mask)
        b = model(xg, mask)
        c = model(xg)
    assert torch.equal(xg, x_copy)
    assert torch.equal(a, b) and torch.equal(a, c)
    assert a.data_ptr() != b.data_ptr()
    assert len(model._graph_cache) == 2  # all_true and none keys
    model.use_cuda_graphs = False
    with torch.inference_mode():
        e = model(xg)
    assert torch.equal(a, e)  # graph replay == the same kernels run eagerly
    _check(om.forward(p, cfg, x), a)


def test_graphs_keep_their_splitk_workspace():
    """Two few-row shapes captured one after the other: the second needs a
    larger split-K workspace, which replaces the model's current one. The
    first graph must keep replaying into the workspace it was captured with,
    never into memory the allocator has since handed to another tensor."""
    cfg = NAMED_CONFIGS["c2"]
    p, _, model = _build(cfg)
    g = torch.Generator().manual_seed(5)
    x_small = torch.randn(1, 32, cfg.d_model, generator=g).cuda()
    x_big = torch.randn(2, 64, cfg.d_model, generator=g).cuda()
    with torch.inference_mode():
        a1 = model(x_small)
        ws_small = model._splitk_ws
        b1 = model(x_big)
        assert model._splitk_ws is not ws_small and model._splitk_ws.numel() > ws_small.numel()
        n_small = ws_small.numel()
        del ws_small
        # tensors of the old workspace's size: if it had been freed, one of
        # them would now sit on its memory
        sentinels = [torch.full((n_small,), 7, dtype=torch.uint8, device="cuda") for _ in range(8)]
        a2 = model(x_small)
        b2 = model(x_big)
        torch.cuda.synchronize()
    for s in sentinels:
        assert bool((s == 7).all()), "a graph replay wrote into memory it does not own"
    assert torch.equal(a1, a2) and torch.equal(b1, b2)
    small_cfg = TransformerConfig(1, 32, cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers, cfg.causal)
    big_cfg = TransformerConfig(2, 64, cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers, cfg.causal)
    _check(om.forward(p, small_cfg, x_small.cpu()), a2)
    _check(om.forward(p, big_cfg, x_big.cpu()), b2)


@pytest.mark.parametrize("masked", [False, True])
def test_chunked_ffn_is_bit_identical(masked):
    """With the FFN budget forced low, the FFN runs over row chunks (5 x 256
    and 120 rows); every GEMM row is computed the same way whatever the row
    count, so the output equals the unchunked forward bit for bit, and both
    pass the gate against the oracle. (1400 rows: enough that the unchunked
    FFN-out does not take the few-row split-K form, whose fixed-order sum
    of K parts is a different rounding.)"""
    cfg = TransformerConfig(2, 700, 256, 4, 1024, 2, False)
    p, x, model = _build(cfg, seed=3)
    mask = om.padded_mask(cfg, 0.3, 11) if masked else None
    if masked:
        x = x.masked_fill(~mask[..., None], 0)
    xg, mg = x.cuda(), (mask.cuda() if masked else None)
    with torch.inference_mode():
        whole = model(xg, mg)
        model.ffn_chunk_budget_bytes = 300 * cfg.ffn_dim * 2
        chunked = model(xg, mg)
    assert torch.equal(whole, chunked)
    _check(om.forward(p, cfg, x, mask), chunked)


@pytest.mark.parametrize("masked", [False, True])
def test_overlapped_layernorm_is_bit_identical(masked):
    """The LayerNorm sites that start under their residual GEMM's tail (ready
    counters) give the same bits as the ones run after the GEMM, in a graph
    and eagerly, and the forward passes the gate."""
    cfg = TransformerConfig(4, 1024, 1024, 16, 4096, 2, True)
    p, x, model = _build(cfg, seed=9)
    mask = om.padded_mask(cfg, 0.3, 5) if masked else None
    if masked:
        x = x.masked_fill(~mask[..., None], 0)
    xg, mg = x.cuda(), (mask.cuda() if masked else None)
    with torch.inference_mode():
        a = model(xg, mg)
        model.overlap_ln = False
        b = model(xg, mg)
        model.use_cuda_graphs = False
        model.overlap_ln = True
        c = model(xg, mg)
        d = model(xg, mg)
    assert torch.equal(a, b) and torch.equal(a, c) and torch.equal(a, d)
    _check(om.forward(p, cfg, x, mask), a)


def test_weight_reload_invalidates_caches():
    cfg = NAMED_CONFIGS["c1"]
    p, x, model = _build(cfg)
    with torch.inference_mode():
        a = model(x.cuda())
    p2, _ = om.seeded_case(cfg, 1)
    model.load_state_dict(p2)
    with torch.inference_mode():
        b = model(x.cuda())
    _check(om.forward(p2, cfg, x), b)
    assert not torch.equal(a, b)


def test_errors_are_loud():
    cfg = TransformerConfig(1, 64, 128, 4, 256, 1, False)  # head_dim 32: no kernel
    model = UserOptimizedTransformer(cfg).cuda()
    with pytest.raises(TfError):
        model(torch.randn(1, 64, 128, device="cuda"))
    with pytest.raises(RuntimeError):
        UserOptimizedTransformer(NAMED_CONFIGS["c1"])(torch.randn(2, 128, 256))


def _gpu_oracle(p, cfg, x, **kw):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    pg = {k: v.cuda() for k, v in p.items()}
    with torch.inference_mode():
        return om.forward(pg, cfg, x.cuda(), **kw)


@pytest.mark.parametrize("name,kw", [
    ("c3", {}),
    ("c4", {"query_tile": 512, "ffn_row_chunk": 32768}),
    ("c5", {"query_tile": 1024, "ffn_row_chunk": 32768}),
])
def test_large_configs(name, kw):
    cfg = NAMED_CONFIGS[name]
    p, x, model = _build(cfg)
    with torch.inference_mode():
        out = model(x.cuda())
    del model
    ref = _gpu_oracle(p, cfg, x, **kw)
    _check(ref, out)


def test_c5_causal():
    cfg = TransformerConfig(1, 100000, 1024, 16, 4096, 4, True)
    p, x, model = _build(cfg)
    with torch.inference_mode():
        out = model(x.cuda())
    del model
    ref = _gpu_oracle(p, cfg, x, query_tile=1024, ffn_row_chunk=32768)
    _check(ref, out)
