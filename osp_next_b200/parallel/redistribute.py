"""Residual-stream redistribution between token layouts across ranks.

This is the Skiparse-SP (SSP) exchange of the reference
(skiparse_func.py:58-139: local permute → one all_to_all_single → permute,
autograd-symmetric), generalised to any pair of layouts (Token↔Group between
sparse blocks, dense↔sparse at the boundaries, where the reference uses an
all-gather and a narrow, osp_next.py:184-189, 1290-1331).  Rows are sent in the
order of their destination row, so the receiver places them with one index
copy and no metadata.  The c10d path here is the portable one (Gloo tests, NCCL
oracle); the fused path stores rows straight into peer buffers from the FFN-down
GEMM epilogue (:mod:`osp_next_b200.parallel.p2p`).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.layout import Redistribution, make_layout, owner_map
from .comm import _a2a_rows


def _to(t, device):
    return t.to(device) if t.device != device else t


def _forward(x: torch.Tensor, rd: Redistribution, group) -> torch.Tensor:
    B, n, C = x.shape
    dev = x.device
    send = x[:, _to(rd.send_rows, dev)].transpose(0, 1).contiguous()          # [Σsend, B, C]
    recv = _a2a_rows(send, rd.send_counts, rd.recv_counts, group)            # [Σrecv, B, C]
    out = x.new_empty(B, rd.n_out, C)
    out[:, _to(rd.recv_rows, dev)] = recv.transpose(0, 1)
    return out


def _backward(g: torch.Tensor, rd: Redistribution, n_in: int, group) -> torch.Tensor:
    B, _, C = g.shape
    dev = g.device
    send = g[:, _to(rd.recv_rows, dev)].transpose(0, 1).contiguous()
    recv = _a2a_rows(send, rd.recv_counts, rd.send_counts, group)
    out = g.new_zeros(B, n_in, C)
    out.index_add_(1, _to(rd.send_rows, dev), recv.transpose(0, 1))     # replicas' grads sum
    return out


class _Redistribute(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, rd, group):
        ctx.rd, ctx.group, ctx.n_in = rd, group, x.shape[1]
        return _forward(x, rd, group)

    @staticmethod
    def backward(ctx, g):
        return _backward(g.contiguous(), ctx.rd, ctx.n_in, ctx.group), None, None


def redistribute(x: torch.Tensor, rd: Redistribution, group) -> torch.Tensor:
    return _Redistribute.apply(x, rd, group)


def gather_natural(x: torch.Tensor, kind: str, grid, P: int, spec, group) -> torch.Tensor:
    """Every rank gets the full sequence in natural order (reference postprocess
    all-gather, osp_next.py:382-424).  Backward keeps the reference's SUM
    semantics: each rank's full-output gradient flows back to the owner rows."""
    from .comm import all_gather
    lay = make_layout(kind, grid, P, spec)
    N = grid[0] * grid[1] * grid[2]
    owner, _ = owner_map(kind, grid, P, spec)
    # only owners contribute (dense replicas would double count)
    sizes, idx = [], []
    for r in range(spec.world):
        from ..models.layout import ParallelSpec
        l_r = make_layout(kind, grid, P, ParallelSpec(spec.ssp, spec.ulysses, spec.full_sp, r))
        mine = owner[l_r.tokens] == r
        sizes.append(int(mine.sum()))
        idx.append(l_r.tokens[mine])
    my_mask = (owner[lay.tokens] == spec.rank).to(x.device)
    xs = x[:, my_mask] if not bool(my_mask.all()) else x
    full = all_gather(xs, dim=1, group=group, sizes=sizes)
    order = torch.cat(idx).to(x.device)
    out = torch.empty(x.shape[0], N, x.shape[2], dtype=x.dtype, device=x.device)
    # differentiable placement
    out = out.index_copy(1, order, full) if not torch.is_grad_enabled() else \
        torch.zeros(x.shape[0], N, x.shape[2], dtype=x.dtype, device=x.device).index_add(1, order, full)
    return out
