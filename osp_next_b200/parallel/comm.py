"""Differentiable collectives used by the DiT (c10d: NCCL on GPU, Gloo on CPU).

Reference counterparts: ospnext/distributed/communication.py — Ulysses 4-D
all-to-all with uneven shard lengths (21-160), all-gather whose backward is a
reduce-scatter with SUM (171-231, which makes per-rank weight gradients sum to
``sp_size ×`` the single-rank gradient — kept here), all_to_all_single (240-315).
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist


def _a2a_rows(x: torch.Tensor, send_counts: List[int], recv_counts: List[int], group) -> torch.Tensor:
    """all_to_all_single over dim 0 with uneven splits."""
    out = x.new_empty((sum(recv_counts),) + tuple(x.shape[1:]))
    dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=group)
    return out


class _UlyssesA2A(torch.autograd.Function):
    """[B, n_r, H, D] (rows of rank r) ⇄ [B, Σn, H/S, D] (all rows, heads of rank r)."""

    @staticmethod
    def forward(ctx, x, group, splits, scatter_heads):
        ctx.group, ctx.splits, ctx.scatter = group, splits, scatter_heads
        return _ulysses(x, group, splits, scatter_heads)

    @staticmethod
    def backward(ctx, g):
        return _ulysses(g.contiguous(), ctx.group, ctx.splits, not ctx.scatter), None, None, None


def _ulysses(x, group, splits, scatter_heads):
    S = dist.get_world_size(group)
    r = dist.get_rank(group)
    if scatter_heads:
        B, n, H, D = x.shape
        hs = H // S
        # send block j = my rows, heads of rank j → [S, B, n, hs, D]
        send = x.view(B, n, S, hs, D).permute(2, 0, 1, 3, 4).contiguous()
        send_counts = [B * n * hs * D] * S
        recv_counts = [B * splits[j] * hs * D for j in range(S)]
        out = _a2a_rows(send.view(-1), send_counts, recv_counts, group)
        parts = torch.split(out, recv_counts)
        parts = [p.view(B, splits[j], hs, D) for j, p in enumerate(parts)]
        return torch.cat(parts, dim=1)
    B, N, hs, D = x.shape
    H = hs * S
    n = splits[r]
    chunks = torch.split(x, splits, dim=1)                       # rows of rank j, my heads
    send = torch.cat([c.reshape(-1) for c in chunks])
    send_counts = [B * splits[j] * hs * D for j in range(S)]
    recv_counts = [B * n * hs * D] * S
    out = _a2a_rows(send, send_counts, recv_counts, group)
    out = out.view(S, B, n, hs, D).permute(1, 2, 0, 3, 4).reshape(B, n, H, D)
    return out


def ulysses_all_to_all(x, group, splits, scatter_heads: bool):
    if group is None or dist.get_world_size(group) == 1:
        return x
    return _UlyssesA2A.apply(x, group, list(splits), scatter_heads)


class _AllGather(torch.autograd.Function):
    """Gather along ``dim`` (uneven sizes allowed); backward reduce-scatters with SUM."""

    @staticmethod
    def forward(ctx, x, dim, group, sizes):
        ctx.dim, ctx.group, ctx.sizes = dim, group, sizes
        xs = x.movedim(dim, 0).contiguous()
        parts = [xs.new_empty((s,) + tuple(xs.shape[1:])) for s in sizes]
        if len(set(sizes)) == 1:
            dist.all_gather(parts, xs, group=group)
        else:
            m = max(sizes)
            pad = xs.new_zeros((m,) + tuple(xs.shape[1:]))
            pad[: xs.shape[0]] = xs
            full = [xs.new_empty(pad.shape) for _ in sizes]
            dist.all_gather(full, pad, group=group)
            parts = [f[:s] for f, s in zip(full, sizes)]
        return torch.cat(parts, 0).movedim(0, dim)

    @staticmethod
    def backward(ctx, g):
        gs = g.movedim(ctx.dim, 0).contiguous()
        parts = list(torch.split(gs, ctx.sizes))
        r = dist.get_rank(ctx.group)
        out = torch.empty_like(parts[r])
        if len(set(ctx.sizes)) == 1:
            dist.reduce_scatter(out, [p.contiguous() for p in parts], op=dist.ReduceOp.SUM, group=ctx.group)
        else:
            # uneven: all-reduce then slice (rare path: boundary gathers of odd grids)
            full = gs.clone()
            dist.all_reduce(full, group=ctx.group)
            out = torch.split(full, ctx.sizes)[r].contiguous()
        return out.movedim(0, ctx.dim), None, None, None


def all_gather(x, dim: int = 1, group=None, sizes: Optional[List[int]] = None):
    if group is None or dist.get_world_size(group) == 1:
        return x
    if sizes is None:
        sizes = gather_sizes(x.shape[dim], group)
    return _AllGather.apply(x, dim, group, list(sizes))


def gather_sizes(n: int, group) -> List[int]:
    """All ranks' lengths (1-element tensors: Gloo rejects 0-dim all_gather_into_tensor)."""
    S = dist.get_world_size(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([n], dtype=torch.int64, device=dev)
    out = [torch.empty_like(t) for _ in range(S)]
    dist.all_gather(out, t, group=group)
    return [int(o.item()) for o in out]


class _AllToAllSingle(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_counts, recv_counts, group):
        ctx.sc, ctx.rc, ctx.group = send_counts, recv_counts, group
        return _a2a_rows(x, send_counts, recv_counts, group)

    @staticmethod
    def backward(ctx, g):
        return _a2a_rows(g.contiguous(), ctx.rc, ctx.sc, ctx.group), None, None, None


def all_to_all_single(x, send_counts, recv_counts, group):
    return _AllToAllSingle.apply(x, list(send_counts), list(recv_counts), group)
