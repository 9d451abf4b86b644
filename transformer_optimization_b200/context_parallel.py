"""Context parallelism: one sequence sharded over the ranks of a process group.

The reference has no multi-GPU code; for sequences too long for one device it
streams shards through host memory (torch_transformer_benchmark.py:4400-4531,
4686-4771). Here the sequence stays resident and is split over GPUs instead:
each rank owns one or more token segments of the global sequence (its
"layout" entry) and runs every token-wise op (LayerNorm, the four GEMMs,
GELU, residual adds) on its own rows. Attention is the one exchange step: a
ring.

Layouts (per rank: a list of (global start, length) segments, concatenated
in that order into the rank's local rows):
  * contiguous: rank r owns shard_bounds(S, n)[r] (non-causal attention costs
    the same on every rank);
  * zigzag: the sequence is cut into 2n chunks and rank r owns chunks r and
    2n-1-r, so under a causal mask every rank has the same amount of work
    (with contiguous shards rank r would compute r+1 of the n key blocks).

Ring attention (per layer). Each rank packs its K|V rows into a contiguous
buffer; for step t = 0 .. n-1 it holds the K|V rows that started on rank
(r - t) mod n, computes flash attention of each of its query segments
against each key segment of that block (global token positions make the
causal mask exact; a segment pair entirely above the diagonal is skipped),
and merges each partial result into the running (O, lse) of its query
segment by log-sum-exp. While step t computes, the block moves one hop (send
to r+1, receive from r-1) into the second buffer, so the NVLink transfer
overlaps the tensor-core work. Remote blocks land in this GPU's own memory
before any kernel reads them. The buffers are kept across layers and calls.

Failure handling: ranks that stop answering make their peers fail instead of
hanging. With `deadline_s` set, the host waits at most that long for each
forward's ring (CPU tensors: every exchange; CUDA tensors: the end of the
forward, by polling an event) and then aborts the group's communicators and
raises RingTimeout. Without it the process group's own timeout applies.

NCCL's send/recv kernels need SMs of their own; while a flash kernel keeps
every SM busy they only get one when a flash CTA exits, and at 8 ranks a
51 MB K|V step then took longer than the flash work it should hide behind.
Give the group high-priority NCCL streams (high_priority_nccl_options(); the
block scheduler then runs NCCL's CTAs first when an SM frees up).

The attention arithmetic is behind a small backend interface: the product
uses `CudaAttentionBackend` (the sm_100a flash and merge kernels); the CPU
tests drive the same ring over gloo with a host backend.
"""

from __future__ import annotations

import datetime
import time
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import kernels

Segment = Tuple[int, int]


class RingTimeout(RuntimeError):
    """A ring exchange did not complete within the host deadline; the
    group's communicators have been aborted."""


def high_priority_nccl_options():
    """Process-group options for the ring: NCCL on high-priority streams
    (pass as pg_options to init_process_group or new_group)."""
    return dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)


def shard_bounds(seq_len: int, world: int) -> List[Segment]:
    """Contiguous (start, length) per rank; the first seq_len % world ranks
    get one extra token."""
    base, rem = divmod(seq_len, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < rem else 0)
        out.append((start, n))
        start += n
    return out


def contiguous_layout(seq_len: int, world: int) -> List[List[Segment]]:
    return [[b] for b in shard_bounds(seq_len, world)]


def zigzag_layout(seq_len: int, world: int) -> List[List[Segment]]:
    """2*world chunks (shard_bounds of the sequence over 2*world); rank r owns
    chunks r and 2*world-1-r, in that order."""
    chunks = shard_bounds(seq_len, 2 * world)
    return [[chunks[r], chunks[2 * world - 1 - r]] for r in range(world)]


def as_layout(bounds_or_layout) -> List[List[Segment]]:
    """Accept either a per-rank list of (start, length) (contiguous shards)
    or a per-rank list of segment lists."""
    out = []
    for entry in bounds_or_layout:
        if len(entry) == 2 and all(isinstance(v, int) for v in entry):
            out.append([(int(entry[0]), int(entry[1]))])
        else:
            out.append([(int(s), int(n)) for s, n in entry])
    return out


def local_length(segments: Sequence[Segment]) -> int:
    return sum(n for _, n in segments)


def local_positions(segments: Sequence[Segment]) -> torch.Tensor:
    """Global token index of each local row."""
    return torch.cat([torch.arange(s, s + n) for s, n in segments]) if segments else torch.zeros(0, dtype=torch.long)


def causal_work(layout: Sequence[Sequence[Segment]]) -> List[int]:
    """Query-key pairs each rank evaluates under a causal mask (for load
    balance checks): sum over its query tokens of (global position + 1)."""
    return [sum((s + n) * (s + n + 1) // 2 - s * (s + 1) // 2 for s, n in segs) for segs in layout]


def ring_sources(rank: int, world: int) -> List[int]:
    """Origin rank of the K/V block a rank holds at each ring step."""
    return [(rank - t) % world for t in range(world)]


class CudaAttentionBackend:
    """Block attention and merge on the B200 kernels. With `timeline` set to
    a list, every merge launch is bracketed by CUDA events on the current
    stream and recorded as ("merge", start, end)."""

    def __init__(self):
        self.timeline: Optional[list] = None

    def block(self, q, k, v, heads, scale, causal, q_pos0, k_pos0, key_valid, first, o_acc, lse_acc, o_part,
              lse_part):
        if first:
            kernels.flash_attention(q, k, v, heads, scale, causal=causal, key_valid=key_valid, q_pos0=q_pos0,
                                    k_pos0=k_pos0, out=o_acc, out_dtype=torch.float32, lse=lse_acc)
        else:
            kernels.flash_attention(q, k, v, heads, scale, causal=causal, key_valid=key_valid, q_pos0=q_pos0,
                                    k_pos0=k_pos0, out=o_part, out_dtype=torch.float32, lse=lse_part)
            if self.timeline is not None:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                kernels.attn_merge(o_acc, lse_acc, o_part, lse_part, heads)
                e.record()
                self.timeline.append(("merge", s, e))
            else:
                kernels.attn_merge(o_acc, lse_acc, o_part, lse_part, heads)

    def finish(self, o_acc, out16):
        out16.copy_(o_acc)


class RingAttention:
    """Ring attention over `group` (all ranks call it together, same shapes
    except the local sequence length)."""

    def __init__(self, group=None, backend=None, deadline_s: Optional[float] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.backend = backend if backend is not None else CudaAttentionBackend()
        self.deadline_s = deadline_s
        self._peer_next = dist.get_global_rank(group, (self.rank + 1) % self.world) if group else (self.rank + 1) % self.world
        self._peer_prev = dist.get_global_rank(group, (self.rank - 1) % self.world) if group else (self.rank - 1) % self.world
        self._buffers: Dict[Tuple, Tuple] = {}
        # with a list here, each ring step's block computation and exposed
        # exchange wait are bracketed by CUDA events: ("block", s, e),
        # ("wait", s, e) (and the backend's ("merge", s, e))
        self.timeline: Optional[list] = None
        self._t_deadline: Optional[float] = None

    def _get_buffers(self, b, s_max, s_loc, d, heads, seg_lens, dt, dev):
        key = (b, s_max, s_loc, d, heads, tuple(seg_lens), dt, dev)
        bufs = self._buffers.get(key)
        if bufs is None:
            n = self.world
            kv = [torch.empty(b, s_max, 2 * d, dtype=dt, device=dev) for _ in range(2 if n > 1 else 1)]
            o_acc = torch.empty(b, s_loc, d, dtype=torch.float32, device=dev)
            o_part = torch.empty_like(o_acc)
            lse_acc = [torch.empty(b, heads, L, dtype=torch.float32, device=dev) for L in seg_lens]
            lse_part = [torch.empty_like(t) for t in lse_acc]
            self._buffers.clear()  # one shape at a time
            bufs = self._buffers[key] = (kv, o_acc, o_part, lse_acc, lse_part)
        return bufs

    def _wait(self, reqs, on_cuda: bool) -> None:
        """Complete this step's exchange. CUDA tensors: the current stream
        waits for it (no host block). CPU tensors with a deadline: the host
        waits at most until the deadline, then aborts and raises."""
        for r in reqs:
            if self._t_deadline is not None and not on_cuda:
                left = self._t_deadline - time.monotonic()
                try:
                    r.wait(datetime.timedelta(seconds=max(left, 0.001)))
                except Exception as exc:
                    self.abort()
                    raise RingTimeout(f"rank {self.rank}: ring exchange not done within {self.deadline_s} s "
                                      f"({exc})") from exc
            else:
                r.wait()

    def abort(self) -> None:
        """Abort the group's communicators (ends any exchange still pending
        on them); the group cannot be used afterwards."""
        try:
            dist.distributed_c10d._abort_process_group(self.group)
        except Exception:
            pass

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float,
                 causal: bool, layout, out16: torch.Tensor,
                 key_valid_full: Optional[torch.Tensor] = None) -> torch.Tensor:
        """q, k, v: this rank's [B, S_loc, D] (any pitch, unit inner stride),
        rows in the order of this rank's segments; layout: per-rank segment
        lists (or contiguous shard_bounds); out16: [B, S_loc, D] receives the
        attention output; key_valid_full: bool [B, S] or None."""
        layout = as_layout(layout)
        b, s_loc, d = q.shape
        n = self.world
        segs = layout[self.rank]
        if local_length(segs) != s_loc:
            raise ValueError(f"rank {self.rank}: {s_loc} local rows but the layout gives {local_length(segs)}")
        s_max = max(local_length(r) for r in layout)
        dev = q.device
        seg_lens = [length for _, length in segs]
        kv, o_acc, o_part, lse_acc, lse_part = self._get_buffers(b, s_max, s_loc, d, heads, seg_lens, k.dtype, dev)
        kv[0][:, :s_loc, :d].copy_(k)
        kv[0][:, :s_loc, d:].copy_(v)
        if self.deadline_s is not None:
            self._t_deadline = time.monotonic() + self.deadline_s
        q_off = [0]
        for length in seg_lens:
            q_off.append(q_off[-1] + length)
        o_acc_v = [o_acc[:, q_off[i]:q_off[i + 1]] for i in range(len(segs))]
        o_part_v = [o_part[:, q_off[i]:q_off[i + 1]] for i in range(len(segs))]
        first = [True] * len(segs)
        tl = self.timeline
        if hasattr(self.backend, "timeline"):
            self.backend.timeline = tl
        for t, src in enumerate(ring_sources(self.rank, n)):
            cur = kv[t % 2]
            reqs = []
            if t < n - 1:
                ops = [dist.P2POp(dist.isend, cur, self._peer_next, self.group),
                       dist.P2POp(dist.irecv, kv[(t + 1) % 2], self._peer_prev, self.group)]
                reqs = dist.batch_isend_irecv(ops)
            if tl is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev0.record()
            k_off = 0
            for k_pos0, k_len in layout[src]:
                if k_len == 0:
                    continue
                kk = cur[:, k_off:k_off + k_len, :d]
                vv = cur[:, k_off:k_off + k_len, d:]
                kv_mask = key_valid_full[:, k_pos0:k_pos0 + k_len] if key_valid_full is not None else None
                for i, (q_pos0, q_len) in enumerate(segs):
                    if q_len == 0 or (causal and k_pos0 > q_pos0 + q_len - 1):
                        continue
                    self.backend.block(q[:, q_off[i]:q_off[i + 1]], kk, vv, heads, scale, causal, q_pos0, k_pos0,
                                       kv_mask, first[i], o_acc_v[i], lse_acc[i], o_part_v[i], lse_part[i])
                    first[i] = False
                k_off += k_len
            if tl is not None:
                ev1 = torch.cuda.Event(enable_timing=True)
                ev1.record()
                tl.append(("block", ev0, ev1))
            self._wait(reqs, cur.is_cuda)
            if tl is not None:
                ev2 = torch.cuda.Event(enable_timing=True)
                ev2.record()
                tl.append(("wait", ev1, ev2))
        for i in range(len(segs)):
            if first[i]:  # every key of every block was masked for these queries
                o_acc_v[i].zero_()
        self.backend.finish(o_acc, out16)
        return out16


class ContextParallelTransformer:
    """Runs a UserOptimizedTransformer with its sequence sharded over `group`.

    forward(x_local, valid_local=None, layout=None) takes this rank's
    [B, S_loc, D] fp32 rows (its layout segments, concatenated) and returns
    the matching rows of the output. layout: per-rank segment lists
    (contiguous_layout / zigzag_layout) or contiguous shard_bounds; None =
    contiguous shards of the gathered local lengths. Same arithmetic as the
    single-GPU forward, with the attention of every layer done by
    RingAttention."""

    def __init__(self, model, group=None, backend=None, deadline_s: Optional[float] = None):
        self.model = model
        self.group = group
        self.ring = RingAttention(group, backend, deadline_s)
        self.deadline_s = deadline_s
        self._bufs: Dict[Tuple, Tuple] = {}

    def _gather_lengths(self, s_loc: int, device) -> List[int]:
        t = torch.tensor([s_loc], dtype=torch.int64, device=device)
        out = [torch.zeros_like(t) for _ in range(self.ring.world)]
        dist.all_gather(out, t, group=self.group)
        return [int(v.item()) for v in out]

    def _gather_mask(self, valid_local, layout, b, dev):
        lens = [local_length(s) for s in layout]
        parts = [torch.zeros(b, n, dtype=torch.bool, device=dev) for n in lens]
        dist.all_gather(parts, valid_local.contiguous(), group=self.group)
        total = sum(lens)
        full = torch.zeros(b, total, dtype=torch.bool, device=dev)
        for segs, part in zip(layout, parts):
            off = 0
            for s, n in segs:
                full[:, s:s + n] = part[:, off:off + n]
                off += n
        return full

    def _buffers(self, b, s_loc, d, f, dev):
        key = (b, s_loc, d, f, dev)
        bufs = self._bufs.get(key)
        if bufs is None:
            self._bufs.clear()
            bufs = self._bufs[key] = (torch.empty(b, s_loc, d, dtype=torch.float32, device=dev),
                                      torch.empty(b, s_loc, d, dtype=torch.float16, device=dev),
                                      torch.empty(b, s_loc, 3 * d, dtype=torch.float16, device=dev),
                                      torch.empty(b, s_loc, d, dtype=torch.float16, device=dev),
                                      torch.empty(b, s_loc, f, dtype=torch.float16, device=dev))
        return bufs

    def _await(self, dev) -> None:
        """Host deadline on the forward's device work (CUDA tensors)."""
        ev = torch.cuda.Event()
        ev.record()
        t_end = time.monotonic() + self.deadline_s
        while not ev.query():
            if time.monotonic() > t_end:
                self.ring.abort()
                raise RingTimeout(f"rank {self.ring.rank}: context-parallel forward not done within "
                                  f"{self.deadline_s} s; communicators aborted")
            time.sleep(0.0002)

    def forward(self, x_local: torch.Tensor, valid_local: Optional[torch.Tensor] = None,
                layout=None, bounds=None) -> torch.Tensor:
        m = self.model
        cfg = m.config
        if not x_local.is_cuda:
            raise RuntimeError("ContextParallelTransformer needs CUDA tensors (no CPU path)")
        if x_local.dtype != torch.float32 or m.final_norm.weight.dtype != torch.float32:
            raise NotImplementedError("context parallelism runs the fp32 model (fp32 ring merge)")
        x_local = x_local.contiguous()
        b, s_loc, d = x_local.shape
        if layout is None:
            layout = bounds
        if layout is None:
            lens = self._gather_lengths(s_loc, x_local.device)
            starts = [sum(lens[:i]) for i in range(len(lens))]
            layout = list(zip(starts, lens))
        layout = as_layout(layout)
        dev = x_local.device
        mask_full = None
        vflat = None
        if valid_local is not None:
            mask_full = self._gather_mask(valid_local, layout, b, dev)
            if bool(mask_full.all()):
                mask_full = None
            else:
                vflat = valid_local.reshape(-1).contiguous()
        active = mask_full is not None
        h = cfg.num_heads
        scale = (d // h) ** -0.5
        wts = m._layer_weights()
        x_res, normed, qkv, ctx, hidden = self._buffers(b, s_loc, d, cfg.ffn_dim, dev)
        # residual GEMM -> LayerNorm pairs overlap as in the single-GPU forward
        ready = kernels.ready_counters(b * s_loc, dev) if (m.overlap_ln and d <= 2048) else None
        fn = m.final_norm
        cur = x_local
        out = None
        normed_ready = False
        n_layers = len(m.layers)
        for li, blk in enumerate(m.layers):
            w = wts[li]
            if not normed_ready:
                kernels.ln_residual(cur, None, w.n1w, w.n1b, blk.norm1.eps, normed=normed)
            kernels.linear(normed, w.wqkv, w.bqkv, out=qkv)
            self.ring(qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:], h, scale, cfg.causal, layout, ctx,
                      mask_full)
            cur = kernels.linear_residual(ctx, w.wo, w.bo, cur, x_res, vflat, mask_delta=active, ready=ready)
            if ready is not None:
                kernels.ln_ready(cur, w.n2w, w.n2b, blk.norm2.eps, ready, normed=normed)
            else:
                kernels.ln_residual(cur, None, w.n2w, w.n2b, blk.norm2.eps, normed=normed)
            kernels.linear(normed, w.w1, w.b1, gelu=True, out=hidden)
            kernels.linear_residual(hidden, w.w2, w.b2, cur, x_res, vflat, mask_x=active, w_split=w.split_w2,
                                    ready=ready)
            if ready is None:
                continue
            if li + 1 < n_layers:
                wn, nxt = wts[li + 1], m.layers[li + 1]
                kernels.ln_ready(cur, wn.n1w, wn.n1b, nxt.norm1.eps, ready, normed=normed)
                normed_ready = True
            else:
                out = kernels.ln_ready(cur, fn.weight, fn.bias, fn.eps, ready, vflat, mask_out=active,
                                       out_dtype=torch.float32)
        if out is None:
            _, out = kernels.ln_residual(cur, None, fn.weight, fn.bias, fn.eps, vflat, mask_out=active,
                                         out_dtype=torch.float32)
        if self.deadline_s is not None:
            self._await(dev)
        return out
