"""Context-parallel forward on 2+ B200s (NCCL P2P ring) against the
single-GPU forward of the same model and input, and against the oracle:
contiguous and zigzag layouts, causal and not, with and without a key
padding mask; a second forward reuses the ring's cached buffers.

Skipped on hosts with fewer than two GPUs. Ranks run as child processes
with a short process-group timeout and a join deadline, so a defect ends in
a failure, not a hang.
"""

import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, causal, layout_kind, masked, q):
    try:
        import datetime

        import torch.distributed as dist

        from oracle import reference_model as om
        from transformer_optimization_b200 import TransformerConfig, UserOptimizedTransformer
        from transformer_optimization_b200.context_parallel import (ContextParallelTransformer, contiguous_layout,
                                                                    local_positions, zigzag_layout)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        cfg = TransformerConfig(2 if masked else 1, 3001, 1024, 16, 4096, 2, causal)
        p, x = om.seeded_case(cfg, 3)
        mask = None
        if masked:
            mask = om.padded_mask(cfg, 0.3, 77)
            x = x.masked_fill(~mask[..., None], 0)
        model = UserOptimizedTransformer(cfg)
        model.load_state_dict(p)
        model = model.cuda().eval()
        layout = (zigzag_layout if layout_kind == "zigzag" else contiguous_layout)(cfg.seq_len, world)
        rows = local_positions(layout[rank])
        with torch.inference_mode():
            full = model(x.cuda(), mask.cuda() if masked else None)
            cp = ContextParallelTransformer(model)
            part = cp.forward(x[:, rows].cuda(), mask[:, rows].cuda() if masked else None, layout=layout)
            again = cp.forward(x[:, rows].cuda(), mask[:, rows].cuda() if masked else None, layout=layout)
            torch.cuda.synchronize()
        if not torch.equal(part, again):
            q.put(f"rank {rank}: a second CP forward (cached ring buffers) differs")
        mine = full[:, rows].cpu()
        got = part.cpu()
        r = om.compare_outputs(mine, got, rtol=0.02, atol=0.002)
        if not r.passed or (mine - got).abs().max() > 1e-3:
            q.put(f"rank {rank}: CP vs single-GPU max diff {(mine - got).abs().max().item():.3g}")
        ref = om.forward(p, cfg, x, mask)[:, rows]
        r2 = om.compare_outputs(ref, got, rtol=0.02, atol=0.002)
        if not r2.passed:
            q.put(f"rank {rank}: CP vs oracle failed {r2.failed_elements} max_abs {r2.max_abs_error:.3g}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put(f"rank {rank} raised: {traceback.format_exc(limit=3)}")


@pytest.mark.parametrize("causal,layout_kind,masked", [
    (False, "contiguous", False),
    (True, "contiguous", False),
    (True, "zigzag", False),
    (False, "contiguous", True),
    (True, "zigzag", True),
])
def test_context_parallel_matches_single_gpu(causal, layout_kind, masked):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 2
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, causal, layout_kind, masked, q))
             for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(300)
    hung = [pr for pr in procs if pr.is_alive()]
    for pr in hung:
        pr.kill()
    errs = []
    while not q.empty():
        errs.append(q.get())
    assert not hung, "context-parallel ranks did not finish"
    assert all(pr.exitcode == 0 for pr in procs), [pr.exitcode for pr in procs]
    assert not errs, "\n".join(errs)
