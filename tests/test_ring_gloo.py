"""Context-parallel ring attention on CPU ranks (gloo): the product's ring
driver (transformer_optimization_b200.context_parallel.RingAttention: shard
bounds, step order, P2P double buffering, global causal positions, key
padding, log-sum-exp merge order) with a host attention backend built from
the oracle, against the oracle's attention over the whole sequence.

Layouts: contiguous shards and the zigzag layout that balances causal work
(rank r owns chunks r and 2n-1-r of 2n).

Also the failure paths: a rank that dies before the exchange makes its peers
raise instead of hanging, and a rank that stalls makes its peers give up at
the host deadline (RingTimeout) instead of waiting for the process-group
timeout.
"""

import math
import os
import socket
import time
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_model as om
from transformer_optimization_b200.context_parallel import (RingAttention, RingTimeout, as_layout, causal_work,
                                                            contiguous_layout, local_positions, ring_sources,
                                                            shard_bounds, zigzag_layout)


class HostBackend:
    """Block attention + merge in fp32 on the CPU (test-only stand-in for the
    CUDA kernels)."""

    @staticmethod
    def _split(t, heads):
        b, s, d = t.shape
        return t.reshape(b, s, heads, d // heads).transpose(1, 2)

    def block(self, q, k, v, heads, scale, causal, q_pos0, k_pos0, key_valid, first, o_acc, lse_acc, o_part,
              lse_part):
        out, lse = om.attention_fp16(self._split(q, heads), self._split(k, heads), self._split(v, heads), scale,
                                     causal, key_valid, q_offset=q_pos0 - k_pos0)
        out = out.transpose(1, 2).reshape(o_acc.shape)
        if first:
            o_acc.copy_(out)
            lse_acc.copy_(lse)
            return
        hd = o_acc.shape[-1] // heads
        L = torch.logaddexp(lse_acc, lse)
        wa = torch.where(torch.isneginf(lse_acc), torch.zeros_like(L), torch.exp(lse_acc - L))
        wb = torch.where(torch.isneginf(lse), torch.zeros_like(L), torch.exp(lse - L))
        wa = wa.transpose(1, 2).repeat_interleave(hd, dim=2)
        wb = wb.transpose(1, 2).repeat_interleave(hd, dim=2)
        o_acc.copy_(o_acc * wa + out * wb)
        lse_acc.copy_(torch.where(torch.isneginf(L), L, L))

    def finish(self, o_acc, out16):
        out16.copy_(o_acc)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q_err, layout_kind="contiguous", stall=False):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        b, s, heads, hd, causal, masked, die = case
        d = heads * hd
        g = torch.Generator().manual_seed(123)
        q = torch.randn(b, s, d, generator=g)
        k = torch.randn(b, s, d, generator=g)
        v = torch.randn(b, s, d, generator=g)
        mask = None
        if masked:
            lengths = torch.tensor([s - 7 * (i + 1) for i in range(b)])
            mask = torch.arange(s)[None, :] < lengths[:, None]
        layout = zigzag_layout(s, world) if layout_kind == "zigzag" else contiguous_layout(s, world)
        rows = local_positions(layout[rank])
        n = rows.numel()
        if die and rank == world - 1:
            raise SystemExit(0)  # leaves before the exchange: peers must not hang
        if stall:
            if rank == world - 1:
                time.sleep(8)  # never joins the exchange in time
                raise SystemExit(0)
            ring = RingAttention(None, HostBackend(), deadline_s=2.0)
            out = torch.empty(b, n, d)
            t0 = time.monotonic()
            try:
                ring(q[:, rows], k[:, rows], v[:, rows], heads, hd ** -0.5, causal, layout, out, mask)
                q_err.put(f"rank {rank}: no RingTimeout")
            except RingTimeout:
                q_err.put(f"rank {rank} RingTimeout after {time.monotonic() - t0:.1f} s")
            return
        ring = RingAttention(None, HostBackend())
        out = torch.empty(b, n, d)
        ring(q[:, rows], k[:, rows], v[:, rows], heads, hd ** -0.5, causal, layout, out, mask)
        # a second call reuses the ring's cached buffers
        out2 = torch.empty(b, n, d)
        ring(q[:, rows], k[:, rows], v[:, rows], heads, hd ** -0.5, causal, layout, out2, mask)
        if not torch.equal(out, out2):
            q_err.put(f"rank {rank}: second call differs")
        ref, _ = om.attention_fp16(HostBackend._split(q, heads), HostBackend._split(k, heads),
                                   HostBackend._split(v, heads), hd ** -0.5, causal, mask)
        ref = ref.transpose(1, 2).reshape(b, s, d)[:, rows]
        if not torch.allclose(out, ref, atol=1e-5, rtol=1e-5):
            q_err.put(f"rank {rank}: max diff {(out - ref).abs().max().item()}")
        dist.barrier()
        dist.destroy_process_group()
    except SystemExit:
        raise
    except Exception:
        q_err.put(f"rank {rank} raised: {traceback.format_exc(limit=2)}")


def _run(world, case, timeout=120, layout_kind="contiguous", stall=False):
    ctx = mp.get_context("spawn")
    q_err = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q_err, layout_kind, stall))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not q_err.empty():
        errs.append(q_err.get())
    return errs, alive


@pytest.mark.parametrize("world,case", [
    (2, (2, 96, 2, 16, False, False, False)),
    (2, (1, 101, 2, 16, True, False, False)),
    (3, (2, 100, 3, 8, True, True, False)),
    (3, (1, 64, 2, 8, False, True, False)),
])
def test_ring_matches_full_attention(world, case):
    errs, alive = _run(world, case)
    assert not alive, "ring ranks hung"
    assert not errs, "\n".join(errs)


@pytest.mark.parametrize("world,case", [
    (2, (1, 101, 2, 16, True, False, False)),
    (3, (2, 100, 3, 8, True, True, False)),
    (4, (1, 203, 2, 8, True, False, False)),
    (2, (2, 96, 2, 16, False, True, False)),
])
def test_zigzag_ring_matches_full_attention(world, case):
    errs, alive = _run(world, case, layout_kind="zigzag")
    assert not alive, "ring ranks hung"
    assert not errs, "\n".join(errs)


def test_zigzag_balances_causal_work():
    """Causal attention work per rank: contiguous shards give the last rank
    ~2n/(n+1) of the mean; the zigzag layout is within a chunk's rounding."""
    s = 100000
    for n in (2, 4, 8):
        cont = causal_work(contiguous_layout(s, n))
        zz = causal_work(zigzag_layout(s, n))
        mean = sum(cont) / n
        assert max(cont) / mean > 1.3
        assert max(zz) / min(zz) < 1.001
        assert sum(zz) == sum(cont) == s * (s + 1) // 2
        lay = zigzag_layout(s, n)
        pos = torch.cat([local_positions(segs) for segs in lay])
        assert torch.equal(pos.sort().values, torch.arange(s))  # a partition of the sequence


def test_stalled_rank_hits_the_deadline():
    """The last rank stalls past the deadline: its peers raise RingTimeout
    after ~2 s (the deadline) instead of waiting 20 s for the process-group
    timeout, and nobody hangs."""
    errs, alive = _run(2, (1, 32, 2, 8, False, False, False), timeout=60, stall=True)
    assert not alive, "ranks hung"
    hits = [e for e in errs if "RingTimeout after" in e]
    assert hits, errs
    assert all(float(e.split("after ")[1].split(" s")[0]) < 8.0 for e in hits), hits


def test_dead_rank_is_detected():
    """The last rank exits before the exchange: the others raise (gloo
    connection closed / timeout) instead of hanging."""
    errs, alive = _run(2, (1, 32, 2, 8, False, False, True), timeout=90)
    assert not alive, "surviving ranks hung"
    assert any("rank 0 raised" in e for e in errs), errs


def test_shard_bounds_and_sources():
    assert shard_bounds(100000, 8) == [(i * 12500, 12500) for i in range(8)]
    b = shard_bounds(10, 3)
    assert b == [(0, 4), (4, 3), (7, 3)]
    assert sum(n for _, n in b) == 10
    assert ring_sources(1, 4) == [1, 0, 3, 2]
    assert zigzag_layout(10, 2) == [[(0, 3), (8, 2)], [(3, 3), (6, 2)]]
    assert as_layout(shard_bounds(10, 3)) == [[(0, 4)], [(4, 3)], [(7, 3)]]
    for r in range(5):
        assert sorted(ring_sources(r, 5)) == list(range(5))
