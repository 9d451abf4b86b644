"""The bounded-wait path on a B200, made to run out without a fault.

Every pipeline wait in the GEMM and attention kernels is bounded by wall
time; when one runs out the kernel records a code in the device status word,
drains what it issued and returns (no trap, no hang). This test runs the
library's probe (tf_test_wait_timeout): a wait on an mbarrier that nothing
ever completes, with a 20 us bound, while the probe's own bulk copy is in
flight. It checks that the wait ran out, the copy drained, the status word
carries the probe's code, tf_last_error says so, and that the device then
still computes a correct forward (c1 against the oracle at the reference's
gate).
"""

import pytest
import torch

from oracle import reference_model as om

pytestmark = pytest.mark.gpu


def test_wait_runs_out_and_device_recovers():
    from transformer_optimization_b200 import NAMED_CONFIGS, UserOptimizedTransformer, _abi, kernels
    _abi.load()
    assert _abi.device_status() == 0  # nothing pending from earlier tests
    src = torch.arange(4096, dtype=torch.int32, device="cuda").to(torch.uint8)
    out = kernels.wait_timeout_probe(src, 20_000)
    torch.cuda.synchronize()
    timed_out, drained, last = out.tolist()
    assert timed_out == 1 and drained == 1
    assert last == 4095 % 256  # the copy issued before the wait landed
    code = _abi.device_status()
    assert code == 106
    assert "device code 106" in _abi.load().tf_last_error().decode()
    assert _abi.device_status() == 0  # reading the status clears it

    cfg = NAMED_CONFIGS["c1"]
    p, x = om.seeded_case(cfg, 0)
    model = UserOptimizedTransformer(cfg)
    model.load_state_dict(p, strict=True)
    model = model.cuda().eval()
    with torch.inference_mode():
        y = model(x.cuda())
    torch.cuda.synchronize()
    assert _abi.device_status() == 0
    r = om.compare_outputs(om.forward(p, cfg, x), y.cpu(), rtol=0.02, atol=0.002)
    assert r.passed, (r.failed_elements, r.max_abs_error)
