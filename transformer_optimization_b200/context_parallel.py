"""Context parallelism: one sequence sharded over the ranks of a process group.

The reference has no multi-GPU code; for sequences too long for one device it
streams shards through host memory (torch_transformer_benchmark.py:4400-4531,
4686-4771). Here the sequence stays resident and is split over GPUs instead:
rank r owns the contiguous token range `shard_bounds(S, n)[r]` and runs every
token-wise op (LayerNorm, the four GEMMs, GELU, residual adds) on its own
rows. Attention is the one exchange step: a ring.

Ring attention (per layer). Each rank packs its K|V rows into a contiguous
buffer; for step t = 0 .. n-1 it holds the K|V block that started on rank
(r - t) mod n, computes flash attention of its queries against that block
(global token positions make the causal mask exact), and merges the partial
result into its running (O, lse) by log-sum-exp. While step t computes, the
block moves one hop (send to r+1, receive from r-1) into the second buffer,
so the NVLink transfer overlaps the tensor-core work. Remote blocks land in
this GPU's own memory before any kernel reads them.

The attention arithmetic is behind a small backend interface: the product
uses `CudaAttentionBackend` (the sm_100a flash and merge kernels); the CPU
tests drive the same ring over gloo with a host backend.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import kernels


def shard_bounds(seq_len: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous (start, length) per rank; the first seq_len % world ranks
    get one extra token."""
    base, rem = divmod(seq_len, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < rem else 0)
        out.append((start, n))
        start += n
    return out


def ring_sources(rank: int, world: int) -> List[int]:
    """Origin rank of the K/V block a rank holds at each ring step."""
    return [(rank - t) % world for t in range(world)]


class CudaAttentionBackend:
    """Block attention and merge on the B200 kernels."""

    def block(self, q, k, v, heads, scale, causal, q_pos0, k_pos0, key_valid, first, o_acc, lse_acc,
              o_part, lse_part):
        if first:
            kernels.flash_attention(q, k, v, heads, scale, causal=causal, key_valid=key_valid, q_pos0=q_pos0,
                                    k_pos0=k_pos0, out=o_acc, out_dtype=torch.float32, lse=lse_acc)
        else:
            kernels.flash_attention(q, k, v, heads, scale, causal=causal, key_valid=key_valid, q_pos0=q_pos0,
                                    k_pos0=k_pos0, out=o_part, out_dtype=torch.float32, lse=lse_part)
            kernels.attn_merge(o_acc, lse_acc, o_part, lse_part, heads)

    def finish(self, o_acc, out16):
        out16.copy_(o_acc)


class RingAttention:
    """Ring attention over `group` (all ranks call it together, same shapes
    except the local sequence length)."""

    def __init__(self, group=None, backend=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.backend = backend if backend is not None else CudaAttentionBackend()
        self._peer_next = dist.get_global_rank(group, (self.rank + 1) % self.world) if group else (self.rank + 1) % self.world
        self._peer_prev = dist.get_global_rank(group, (self.rank - 1) % self.world) if group else (self.rank - 1) % self.world

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float,
                 causal: bool, bounds: Sequence[Tuple[int, int]], out16: torch.Tensor,
                 key_valid_full: Optional[torch.Tensor] = None) -> torch.Tensor:
        """q, k, v: this rank's [B, S_loc, D] (any pitch, unit inner stride);
        bounds: shard_bounds of the full sequence; out16: [B, S_loc, D]
        receives the attention output; key_valid_full: bool [B, S] or None."""
        b, s_loc, d = q.shape
        n = self.world
        s_max = max(length for _, length in bounds)
        dev = q.device
        dt = k.dtype
        # contiguous K|V send/receive buffers (double buffered)
        bufs = [torch.empty(b, s_max, 2 * d, dtype=dt, device=dev) for _ in range(2 if n > 1 else 1)]
        bufs[0][:, :s_loc, :d].copy_(k)
        bufs[0][:, :s_loc, d:].copy_(v)
        o_acc = torch.empty(b, s_loc, d, dtype=torch.float32, device=dev)
        lse_acc = torch.empty(b, heads, s_loc, dtype=torch.float32, device=dev)
        o_part = torch.empty_like(o_acc) if n > 1 else None
        lse_part = torch.empty_like(lse_acc) if n > 1 else None
        q_pos0 = bounds[self.rank][0]
        q_last = q_pos0 + s_loc - 1
        first = True
        for t, src in enumerate(ring_sources(self.rank, n)):
            cur = bufs[t % 2]
            reqs = []
            if t < n - 1:
                ops = [dist.P2POp(dist.isend, cur, self._peer_next, self.group),
                       dist.P2POp(dist.irecv, bufs[(t + 1) % 2], self._peer_prev, self.group)]
                reqs = dist.batch_isend_irecv(ops)
            k_pos0, k_len = bounds[src]
            skip = k_len == 0 or (causal and k_pos0 > q_last)
            if not skip:
                kv_mask = None
                if key_valid_full is not None:
                    kv_mask = key_valid_full[:, k_pos0:k_pos0 + k_len]
                self.backend.block(q, cur[:, :k_len, :d], cur[:, :k_len, d:], heads, scale, causal, q_pos0, k_pos0,
                                   kv_mask, first, o_acc, lse_acc, o_part, lse_part)
                first = False
            for r in reqs:
                r.wait()
        if first:  # every key of every block was masked for these queries
            o_acc.zero_()
        self.backend.finish(o_acc, out16)
        return out16


class ContextParallelTransformer:
    """Runs a UserOptimizedTransformer with its sequence sharded over `group`.

    forward(x_local, valid_local=None) takes this rank's [B, S_loc, D] fp32
    slice (shard_bounds of the full length) and returns the matching slice of
    the output. Same arithmetic as the single-GPU forward, with the attention
    of every layer done by RingAttention."""

    def __init__(self, model, group=None, backend=None):
        self.model = model
        self.group = group
        self.ring = RingAttention(group, backend)

    def _gather_lengths(self, s_loc: int, device) -> List[int]:
        t = torch.tensor([s_loc], dtype=torch.int64, device=device)
        out = [torch.zeros_like(t) for _ in range(self.ring.world)]
        dist.all_gather(out, t, group=self.group)
        return [int(v.item()) for v in out]

    def forward(self, x_local: torch.Tensor, valid_local: Optional[torch.Tensor] = None,
                bounds: Optional[Sequence[Tuple[int, int]]] = None) -> torch.Tensor:
        m = self.model
        cfg = m.config
        if not x_local.is_cuda:
            raise RuntimeError("ContextParallelTransformer needs CUDA tensors (no CPU path)")
        if x_local.dtype != torch.float32 or m.final_norm.weight.dtype != torch.float32:
            raise NotImplementedError("context parallelism runs the fp32 model (fp32 ring merge)")
        x_local = x_local.contiguous()
        b, s_loc, d = x_local.shape
        if bounds is None:
            lens = self._gather_lengths(s_loc, x_local.device)
            starts = [sum(lens[:i]) for i in range(len(lens))]
            bounds = list(zip(starts, lens))
        mask_full = None
        vflat = None
        if valid_local is not None:
            parts = [torch.zeros(b, length, dtype=torch.bool, device=x_local.device) for _, length in bounds]
            dist.all_gather(parts, valid_local.contiguous(), group=self.group)
            mask_full = torch.cat(parts, dim=1)
            if bool(mask_full.all()):
                mask_full = None
            else:
                vflat = valid_local.reshape(-1)
        active = mask_full is not None
        h = cfg.num_heads
        scale = (d // h) ** -0.5
        wts = m._layer_weights()
        dev = x_local.device
        x_res = torch.empty(b, s_loc, d, dtype=torch.float32, device=dev)
        normed = torch.empty(b, s_loc, d, dtype=torch.float16, device=dev)
        qkv = torch.empty(b, s_loc, 3 * d, dtype=torch.float16, device=dev)
        ctx = torch.empty(b, s_loc, d, dtype=torch.float16, device=dev)
        hidden = torch.empty(b, s_loc, cfg.ffn_dim, dtype=torch.float16, device=dev)
        cur = x_local
        for li, blk in enumerate(m.layers):
            w = wts[li]
            kernels.ln_residual(cur, None, w.n1w, w.n1b, blk.norm1.eps, normed=normed)
            kernels.linear(normed, w.wqkv, w.bqkv, out=qkv)
            self.ring(qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:], h, scale, cfg.causal, bounds, ctx,
                      mask_full)
            cur = kernels.linear_residual(ctx, w.wo, w.bo, cur, x_res, vflat, mask_delta=active)
            kernels.ln_residual(cur, None, w.n2w, w.n2b, blk.norm2.eps, normed=normed)
            kernels.linear(normed, w.w1, w.b1, gelu=True, out=hidden)
            kernels.linear_residual(hidden, w.w2, w.b2, cur, x_res, vflat, mask_x=active, w_split=w.split_w2)
        fn = m.final_norm
        _, out = kernels.ln_residual(cur, None, fn.weight, fn.bias, fn.eps, vflat, mask_out=active,
                                     out_dtype=torch.float32)
        return out
