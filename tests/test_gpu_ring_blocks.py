"""Context parallelism's attention arithmetic on ONE B200: the sequence of
flash blocks (keys at global positions, causal on global positions, key
padding) and log-sum-exp merges that RingAttention runs on each rank, run here
for every rank of a virtual ring in the order the ring delivers the K/V
blocks (ring_sources), through the same CudaAttentionBackend the ring uses.
Each virtual rank's output must match one flash call over the whole sequence.
The NCCL exchange itself is covered by tests/test_gpu_cp.py (two or more
GPUs) and tests/test_ring_gloo.py (host ranks)."""

import pytest
import torch

from transformer_optimization_b200 import kernels as K
from transformer_optimization_b200.context_parallel import (CudaAttentionBackend, contiguous_layout,
                                                            local_positions, ring_sources, zigzag_layout)

pytestmark = pytest.mark.gpu


def _virtual_rank(q, k, v, heads, scale, causal, key_valid, layout, rank):
    """RingAttention.__call__'s block / merge schedule for `rank`, with each
    step's K/V block taken straight from the full tensors."""
    b, _, d = q.shape
    segs = layout[rank]
    rows = local_positions(segs).to(q.device)
    q_loc = q[:, rows]
    s_loc = q_loc.shape[1]
    q_off = [0]
    for _, n in segs:
        q_off.append(q_off[-1] + n)
    o_acc = torch.empty(b, s_loc, d, dtype=torch.float32, device=q.device)
    o_part = torch.empty_like(o_acc)
    lse_acc = [torch.empty(b, heads, n, dtype=torch.float32, device=q.device) for _, n in segs]
    lse_part = [torch.empty_like(t) for t in lse_acc]
    first = [True] * len(segs)
    backend = CudaAttentionBackend()
    for src in ring_sources(rank, len(layout)):
        for k_pos0, k_len in layout[src]:
            if k_len == 0:
                continue
            kk = k[:, k_pos0:k_pos0 + k_len]
            vv = v[:, k_pos0:k_pos0 + k_len]
            kv_mask = key_valid[:, k_pos0:k_pos0 + k_len] if key_valid is not None else None
            for i, (q_pos0, q_len) in enumerate(segs):
                if q_len == 0 or (causal and k_pos0 > q_pos0 + q_len - 1):
                    continue
                backend.block(q_loc[:, q_off[i]:q_off[i + 1]], kk, vv, heads, scale, causal, q_pos0, k_pos0,
                              kv_mask, first[i], o_acc[:, q_off[i]:q_off[i + 1]], lse_acc[i],
                              o_part[:, q_off[i]:q_off[i + 1]], lse_part[i])
                first[i] = False
    out16 = torch.empty(b, s_loc, d, dtype=torch.float16, device=q.device)
    backend.finish(o_acc, out16)
    return rows, out16


@pytest.mark.parametrize("layout_kind", ["contiguous", "zigzag"])
@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("causal,masked", [(False, False), (True, False), (False, True), (True, True)])
def test_ring_blocks_match_full_attention(layout_kind, world, causal, masked):
    b, s, heads, hd = 2, 3001, 16, 64
    d = heads * hd
    g = torch.Generator().manual_seed(world * 10 + causal * 2 + masked)
    q = (torch.randn(b, s, d, generator=g) * 1.5).half().cuda()
    k = (torch.randn(b, s, d, generator=g) * 1.5).half().cuda()
    v = torch.randn(b, s, d, generator=g).half().cuda()
    key_valid = None
    if masked:
        lengths = torch.tensor([s - 411, s - 1777])
        key_valid = (torch.arange(s)[None, :] < lengths[:, None]).cuda()
    scale = hd ** -0.5
    full, _ = K.flash_attention(q, k, v, heads, scale, causal=causal, key_valid=key_valid)
    layout = (zigzag_layout if layout_kind == "zigzag" else contiguous_layout)(s, world)
    for rank in range(world):
        rows, out = _virtual_rank(q, k, v, heads, scale, causal, key_valid, layout, rank)
        ref = full[:, rows].float()
        err = (out.float() - ref).abs()
        assert torch.all(err <= 1e-2 * ref.abs() + 3e-3), f"rank {rank}: max err {err.max()}"
    from transformer_optimization_b200 import _abi
    assert _abi.device_status() == 0
