"""Varlen pack/unpack of padded token batches (reference: ospnext/utils/padding.py:8-137).

``unpad_input`` packs the valid rows of a ``[B, S, ...]`` batch into ``[nnz, ...]``
and returns the flat row indices plus ``cu_seqlens`` offsets; ``pad_input`` scatters
them back.  Both are differentiable (gather ↔ scatter-add are each other's
adjoints).  The segmented attention kernel consumes ``cu_seqlens`` directly, so the
model itself never pads; these helpers serve callers that hold masked batches.

As in the reference, ``max_seqlen_in_batch`` is the padded length ``S`` (an upper
bound), not the longest valid row.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


class _GatherRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, idx):
        ctx.save_for_backward(idx)
        ctx.n = x.shape[0]
        return x.index_select(0, idx)

    @staticmethod
    def backward(ctx, g):
        (idx,) = ctx.saved_tensors
        out = g.new_zeros((ctx.n,) + tuple(g.shape[1:]))
        out.index_add_(0, idx, g)
        return out, None


class _ScatterRows(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, idx, n):
        ctx.save_for_backward(idx)
        out = x.new_zeros((n,) + tuple(x.shape[1:]))
        out.index_copy_(0, idx, x)
        return out

    @staticmethod
    def backward(ctx, g):
        (idx,) = ctx.saved_tensors
        return g.index_select(0, idx), None, None


def index_first_axis(x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Rows ``x[indices]`` with a scatter-add backward."""
    return _GatherRows.apply(x, indices)


def index_put_first_axis(values: torch.Tensor, indices: torch.Tensor, first_axis_dim: int) -> torch.Tensor:
    """Zero tensor of ``first_axis_dim`` rows with ``values`` at ``indices``."""
    return _ScatterRows.apply(values, indices, int(first_axis_dim))


def unpad_input(hidden_states: torch.Tensor, attention_mask: torch.Tensor):
    """``[B,S,...]`` + mask ``[B,S]`` → (packed ``[nnz,...]``, indices, cu_seqlens int32 [B+1], S)."""
    B, S = attention_mask.shape
    lens = attention_mask.sum(dim=-1, dtype=torch.int32)
    indices = torch.nonzero(attention_mask.reshape(-1), as_tuple=False).reshape(-1)
    cu = F.pad(torch.cumsum(lens, 0, dtype=torch.int32), (1, 0))
    flat = hidden_states.reshape(B * S, *hidden_states.shape[2:])
    return index_first_axis(flat, indices), indices, cu, hidden_states.shape[1]


def pad_input(hidden_states: torch.Tensor, indices: torch.Tensor, batch: int, seqlen: int) -> torch.Tensor:
    """Inverse of :func:`unpad_input`: ``[nnz,...]`` → ``[batch, seqlen, ...]`` (zeros at pads)."""
    out = index_put_first_axis(hidden_states, indices, batch * seqlen)
    return out.view(batch, seqlen, *hidden_states.shape[1:])
