"""tf_gemm_splitk_static: the split-K GEMM with the library's fixed device
scratch in place of a caller workspace (no allocation in the call).

Collected last (file name) so it also runs after every other GPU test in the
same process; it passes alone as well. Two calls in a row must both equal the
workspace entry point tf_gemm_splitk on the same inputs (same kernels, same
split plan, fixed-order reduction: bit-identical), and a call whose partial
sums would exceed the 4 MiB scratch is refused.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(m, k, n, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).half()
    bound = 1 / math.sqrt(k)
    w = ((torch.rand(n, k, generator=g) * 2 - 1) * bound).half()
    b = (torch.rand(n, generator=g) * 2 - 1) * bound
    return a.cuda(), w.cuda(), b.cuda()


def _static(a, w, b, out, gelu, splits):
    from transformer_optimization_b200 import _abi
    m, k = a.shape
    n = w.shape[0]
    _abi.call("tf_gemm_splitk_static", a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), b.data_ptr(),
              out.data_ptr(), out.stride(0), m, n, k, _abi.TF_EPI_BIAS_GELU if gelu else _abi.TF_EPI_BIAS, splits,
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,k,n,gelu,splits", [(64, 2048, 512, False, 0), (64, 512, 2048, True, 0),
                                               (256, 1024, 256, False, 8), (300, 1024, 768, True, 3)])
def test_static_scratch_matches_workspace_entry(m, k, n, gelu, splits):
    from transformer_optimization_b200 import kernels as K
    a, w, b = _inputs(m, k, n, m + k + n)
    ref = K.linear(a, w, b, gelu=gelu, splits=splits)  # tf_gemm_splitk with a torch-allocated workspace
    first = torch.empty(m, n, dtype=torch.float16, device="cuda")
    second = torch.empty(m, n, dtype=torch.float16, device="cuda")
    _static(a, w, b, first, gelu, splits)
    _static(a, w, b, second, gelu, splits)
    torch.cuda.synchronize()
    assert torch.equal(first, ref)
    assert torch.equal(second, ref)


def test_static_scratch_limit():
    from transformer_optimization_b200 import _abi, kernels as K
    m, k, n = 1024, 4096, 1024
    assert K.splitk_workspace_bytes(m, n, k, 4) > 4 << 20
    a, w, b = _inputs(m, k, n, 1)
    out = torch.empty(m, n, dtype=torch.float16, device="cuda")
    with pytest.raises(_abi.TfError, match="scratch"):
        _static(a, w, b, out, False, 4)
