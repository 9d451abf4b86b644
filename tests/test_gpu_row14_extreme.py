"""The reference's hardest published case on one B200: the user matrix's row
14 (run_bench.py user_matrix "14_extreme": batch 32, sequence 100 000, d_model
1024, 16 heads, ffn 1024, 2 layers, causal). The reference streams it on its
16 GB card; here the 13 GB input and ~70 GB of activations fit in HBM and the
forward runs unstreamed.

Batch elements are independent, so parity is checked on two of them (the
first and the last) against the oracle's fp32 query-tiled model run on the
GPU (TF32 off), with the reference's gate; the rest of the output is checked
for finiteness. Inputs are drawn on the GPU from a seeded generator.
"""

import gc

import pytest
import torch

from oracle import reference_model as om
from transformer_optimization_b200 import TransformerConfig, UserOptimizedTransformer

pytestmark = pytest.mark.gpu


def test_row14_extreme():
    gc.collect()
    torch.cuda.empty_cache()  # memory cached by earlier tests in this process
    free, _ = torch.cuda.mem_get_info()
    if free < 120 << 30:
        pytest.skip("needs ~120 GB of free device memory")
    cfg = TransformerConfig(32, 100000, 1024, 16, 1024, 2, True)
    p = om.init_params(cfg, 0)
    model = UserOptimizedTransformer(cfg)
    model.load_state_dict(p, strict=True)
    model = model.cuda().eval()
    g = torch.Generator(device="cuda").manual_seed(14)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, device="cuda", generator=g)
    with torch.inference_mode():
        out = model(x)
    torch.cuda.synchronize()
    del model
    torch.cuda.empty_cache()
    assert out.shape == x.shape and out.dtype == torch.float32
    assert bool(torch.isfinite(out).all())

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    pg = {k: v.cuda() for k, v in p.items()}
    for b in (0, cfg.batch_size - 1):
        with torch.inference_mode():
            ref = om.forward(pg, cfg, x[b:b + 1], query_tile=1024, ffn_row_chunk=32768)
        r = om.compare_outputs(ref.float().cpu(), out[b:b + 1].float().cpu(), rtol=0.02, atol=0.002)
        assert r.passed, (f"batch {b}: {r.failed_elements}/{r.total_elements} failed, "
                          f"max_abs={r.max_abs_error:.3g} at {r.worst_index}")
