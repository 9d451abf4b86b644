"""The reference harness's own accuracy check, run_accuracy_tests
(torch_transformer_benchmark.py:4618-4683), on a B200: for each trial t of
5, generate_random_case with seed 1234 + t on the GPU (oracle.harness_case),
the eager model's output (the oracle's forward, strict fp32 on the GPU), the
optimized model's, and compare_outputs with atol 0.002, rtol 0.02 and zero
failing elements - the harness defaults (torch_transformer_benchmark.py:
5044-5050), with and without key padding, at input scales 1 and 3. The fp32
model is the configuration the gate is defined for; fp16 and bf16 models are
checked the same way in tests/test_gpu_half_models.py.
"""

import pytest
import torch

from oracle import reference_model as om
from transformer_optimization_b200 import NAMED_CONFIGS, TransformerConfig, UserOptimizedTransformer

pytestmark = pytest.mark.gpu
TRIALS, SEED, ATOL, RTOL = 5, 1234, 0.002, 0.02

CONFIGS = {
    "c1": NAMED_CONFIGS["c1"],
    "c1_causal": TransformerConfig(2, 128, 256, 4, 1024, 2, True),
    "c2": NAMED_CONFIGS["c2"],
    "mid_causal": TransformerConfig(4, 512, 512, 8, 2048, 3, True),
}


@pytest.fixture(scope="module", autouse=True)
def strict_fp32():
    old = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


@pytest.mark.parametrize("padding_ratio,input_scale", [(0.0, 1.0), (0.4, 1.0), (0.0, 3.0)])
@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_run_accuracy_tests_protocol(name, padding_ratio, input_scale):
    dtype = torch.float32
    cfg = CONFIGS[name]
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    p = om.init_params(cfg, None)
    model = UserOptimizedTransformer(cfg)
    model.load_state_dict(p, strict=True)
    model = model.to(dev, dtype).eval()
    pg = {k: v.to(dev, dtype) for k, v in p.items()}
    failed = []
    with torch.inference_mode():
        for trial in range(TRIALS):
            x, mask = om.harness_case(cfg, dev, dtype, SEED + trial, padding_ratio, input_scale)
            reference = om.forward(pg, cfg, x, mask)
            candidate = model(x, mask)
            r = om.compare_outputs(reference.float().cpu(), candidate.float().cpu(), rtol=RTOL, atol=ATOL)
            if not r.passed:
                failed.append((trial, r.failed_elements, r.max_abs_error, r.worst_index))
    assert not failed, f"trials failing the harness gate: {failed}"
