"""Training-capable SSP exchange and Ulysses all-to-all over NVLink peer memory.

The reference moves the residual stream between Skiparse layouts with a local permute,
one NCCL ``all_to_all_single`` and another permute, forward and backward
(ospnext/modules/skiparse_func.py:58-139, osp_next.py:887-924), and runs Ulysses as a
4-D all-to-all (ospnext/distributed/communication.py:21-128).  Here each is one staged
pull over the :class:`~osp_next_b200.parallel.p2p.P2PExchange` staging ring:

1. every rank copies its input (contiguous) into its staging slot;
2. one bounded device barrier orders the copies;
3. every rank pulls the chunks of its output from the ranks that hold them
   (``ops.ext().p2p_pull``, a table of (source rank, byte offset) per output chunk built
   once per layout pair on the host), straight into a fresh tensor autograd may keep.

There is no permute pass and no NCCL launch; the backward is the same pull with the
inverse table, and where the forward fanned one row out to several dense-layout replicas,
the backward table lists every replica and the pull sums them in fp32 (the reference's
``index_add`` of replica gradients).  Rows a rank holds only as a replica get zero
gradient, as in the c10d path (:mod:`osp_next_b200.parallel.redistribute`).

The table builders are pure functions of the layouts; :func:`emulate_pull` replays a
table over per-rank byte buffers on the CPU, which is how the host-side logic is tested
without GPUs.
"""
from __future__ import annotations

from functools import lru_cache
from typing import List, Sequence, Tuple

import torch

from .. import ops
from ..models.layout import FULL, ParallelSpec, make_layout, owner_map


def _pad16(n: int) -> int:
    return (n + 15) // 16 * 16


def _spec(spec: ParallelSpec, r: int) -> ParallelSpec:
    return ParallelSpec(spec.ssp, spec.ulysses, spec.full_sp, r)


def _check(off: torch.Tensor, chunk: int):
    if chunk % 16 or bool((off % 16 != 0).any()):
        raise ValueError("p2p pull tables need 16-byte aligned chunks and offsets")


# ----------------------------------------------------------------------------- table builders
@lru_cache(maxsize=128)
def redistribute_tables(ka: str, kb: str, grid: Tuple[int, int, int], P: int, spec: ParallelSpec, B: int,
                        C: int, esz: int, esz_grad: int):
    """Pull tables for moving ``[B, n_a, C]`` rows of layout ``ka`` to ``kb`` on rank ``spec.rank``.

    Forward: every rank stages its ``[B, n_a(r), C]`` input; output row j of batch b comes
    from the owner of its token in layout A.  Backward: every rank stages its gradient
    ``[B, n_b(r), C]`` (``esz_grad`` bytes per element); an A row this rank owns sums the
    gradient of each B rank holding the token (one, or every dense replica); other A rows
    get zeros.  Returns (n_in, n_out, f_rank, f_off, b_rank, b_off, R)."""
    W = spec.world
    la, lb = make_layout(ka, grid, P, spec), make_layout(kb, grid, P, spec)
    n_a = torch.tensor([make_layout(ka, grid, P, _spec(spec, r)).n_local for r in range(W)])
    n_b = torch.tensor([make_layout(kb, grid, P, _spec(spec, r)).n_local for r in range(W)])
    own_a, row_a = owner_map(ka, grid, P, spec)
    own_b, row_b = owner_map(kb, grid, P, spec)
    b = torch.arange(B)[:, None]
    src = own_a[lb.tokens]
    f_rank = src[None, :].expand(B, -1).reshape(-1).to(torch.int32).contiguous()
    f_off = ((b * n_a[src][None, :] + row_a[lb.tokens][None, :]) * (C * esz)).reshape(-1).contiguous()
    # backward sources: the B owner and its replicas r + k·full_sp (dense B), same row
    R = W // spec.full_sp if (kb == FULL or P == 1) else 1
    mine = own_a[la.tokens] == spec.rank
    ranks = torch.stack([own_b[la.tokens] + k * spec.full_sp for k in range(R)], 1)           # [n_a, R]
    rows = row_b[la.tokens][:, None].expand(-1, R)
    ranks = torch.where(mine[:, None], ranks, torch.full_like(ranks, -1))
    b_rank = ranks[None].expand(B, -1, -1).reshape(-1).to(torch.int32).contiguous()
    b_off = ((b[:, :, None] * n_b[ranks.clamp_min(0)][None] + rows[None]) * (C * esz_grad))
    b_off = torch.where(ranks[None] >= 0, b_off, torch.zeros_like(b_off)).reshape(-1).contiguous()
    _check(f_off, C * esz)
    _check(b_off, C * esz_grad)
    return la.n_local, lb.n_local, f_rank, f_off, b_rank, b_off, R


@lru_cache(maxsize=128)
def ulysses_tables(S: int, j: int, base: int, splits: Tuple[int, ...], B: int, H: int, D: int, esz: int,
                   n_t: int, scatter: bool):
    """Pull tables of the Ulysses all-to-all for ``n_t`` tensors staged back to back.

    scatter (rows → heads): member r of the group (global rank ``base + r``) stages
    ``[B, splits[r], H, D]`` per tensor; member ``j`` pulls ``[n_t, B, N, H/S, D]``, the
    chunk (t, b, g) being row g's heads ``j·H/S …`` from the member owning row g.
    gather (heads → rows): every member stages ``[B, N, H/S, D]`` per tensor; member ``j``
    pulls ``[n_t, B, splits[j], H, D]``, the chunk (t, b, i, r) being member r's heads of
    row ``offs[j] + i``.  Returns (rank, off, chunk_bytes)."""
    hs = H // S
    N = sum(splits)
    offs = [0]
    for s in splits:
        offs.append(offs[-1] + s)
    chunk = hs * D * esz
    if scatter:
        size = [_pad16(B * splits[r] * H * D * esz) for r in range(S)]
        g = torch.arange(N)
        owner = torch.bucketize(g, torch.tensor(offs[1:]), right=True)
        row = g - torch.tensor(offs)[owner]
        spl = torch.tensor(splits)[owner]
        sz = torch.tensor(size)[owner]
        t = torch.arange(n_t)[:, None, None]
        bb = torch.arange(B)[None, :, None]
        off = t * sz + ((bb * spl + row) * H + j * hs) * D * esz
        rank = (base + owner)[None, None, :].expand(n_t, B, -1)
    else:
        size = _pad16(B * N * hs * D * esz)
        n = splits[j]
        t = torch.arange(n_t)[:, None, None, None]
        bb = torch.arange(B)[None, :, None, None]
        i = torch.arange(n)[None, None, :, None]
        r = torch.arange(S)[None, None, None, :]
        off = t * size + ((bb * N + offs[j] + i) * hs) * D * esz + 0 * r
        rank = (base + r).expand(n_t, B, n, S)
    off = off.reshape(-1).contiguous()
    _check(off, chunk)
    return rank.reshape(-1).to(torch.int32).contiguous(), off, chunk


# ----------------------------------------------------------------------------- pulls
_DEV = {}


def _dev(t: torch.Tensor, device) -> torch.Tensor:
    key = (id(t), str(device))
    hit = _DEV.get(key)
    if hit is None or hit[0] is not t:
        hit = (t, t.to(device))
        _DEV[key] = hit
    return hit[1]


def _pull(ex, tensors: Sequence[torch.Tensor], out: torch.Tensor, rank, off, R: int, chunk: int, sum_: bool):
    ptrs = ex.stage([t.contiguous() for t in tensors])
    ops.ext().p2p_pull(out, ptrs, _dev(rank, out.device), _dev(off, out.device), R, chunk, sum_)
    return out


def emulate_pull(stages: List[torch.Tensor], rank: torch.Tensor, off: torch.Tensor, R: int, chunk: int,
                 sum_: bool, out: torch.Tensor) -> torch.Tensor:
    """CPU replay of ``p2p_pull`` over per-rank uint8 staging buffers (tests)."""
    flat = out.view(-1).view(torch.uint8)
    n = flat.numel() // chunk
    for u in range(n):
        if not sum_:
            r = int(rank[u])
            piece = stages[r][int(off[u]):int(off[u]) + chunk] if r >= 0 else torch.zeros(chunk, dtype=torch.uint8)
            flat[u * chunk:(u + 1) * chunk] = piece
        else:
            acc = torch.zeros(chunk // 4, dtype=torch.float32)
            for k in range(R):
                r = int(rank[u * R + k])
                if r >= 0:
                    acc += stages[r][int(off[u * R + k]):int(off[u * R + k]) + chunk].view(torch.float32)
            flat[u * chunk:(u + 1) * chunk] = acc.view(torch.uint8)
    return out


def stage_bytes(tensors: Sequence[torch.Tensor]) -> torch.Tensor:
    """The staging slot contents ``P2PExchange.stage`` writes for ``tensors`` (tests)."""
    parts = []
    for t in tensors:
        b = t.contiguous().view(-1).view(torch.uint8)
        parts.append(b)
        pad = _pad16(b.numel()) - b.numel()
        if pad:
            parts.append(torch.zeros(pad, dtype=torch.uint8))
    return torch.cat(parts) if parts else torch.zeros(0, dtype=torch.uint8)


# ----------------------------------------------------------------------------- autograd
class _Redistribute(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, ex, key):
        ka, kb, grid, P, spec = key
        B, _, C = x.shape
        esz_g = 4 if (kb == FULL or P == 1) and spec.world > spec.full_sp else x.element_size()
        n_in, n_out, f_rank, f_off, b_rank, b_off, R = redistribute_tables(
            ka, kb, grid, P, spec, B, C, x.element_size(), esz_g)
        ctx.ex, ctx.tabs, ctx.xdt = ex, (n_in, b_rank, b_off, R, C * esz_g, esz_g), x.dtype
        out = torch.empty(B, n_out, C, dtype=x.dtype, device=x.device)
        return _pull(ex, [x], out, f_rank, f_off, 1, C * x.element_size(), False)

    @staticmethod
    def backward(ctx, g):
        n_in, b_rank, b_off, R, chunk, esz_g = ctx.tabs
        g = g.contiguous()
        if esz_g == 4:
            g = g.float()
        B, _, C = g.shape
        dx = torch.empty(B, n_in, C, dtype=g.dtype, device=g.device)
        _pull(ctx.ex, [g], dx, b_rank, b_off, R, chunk, R > 1)
        return dx.to(ctx.xdt), None, None


def p2p_redistribute(x: torch.Tensor, ka: str, kb: str, grid, P: int, spec: ParallelSpec, ex) -> torch.Tensor:
    """Residual rows of layout ``ka`` → ``kb`` over NVLink (differentiable)."""
    return _Redistribute.apply(x, ex, (ka, kb, tuple(grid), P, spec))


class _UlyssesScatter(torch.autograd.Function):
    """Tensors [B, n_j, H, D] (rows of member j) → [B, N, H/S, D] (all rows, heads of j)."""

    @staticmethod
    def forward(ctx, ex, grp, *ts):
        S, j, base, splits = grp
        B, _, H, D = ts[0].shape
        rank, off, chunk = ulysses_tables(S, j, base, splits, B, H, D, ts[0].element_size(), len(ts), True)
        out = torch.empty(len(ts), B, sum(splits), H // S, D, dtype=ts[0].dtype, device=ts[0].device)
        _pull(ex, ts, out, rank, off, 1, chunk, False)
        ctx.ex, ctx.grp = ex, grp
        return tuple(out.unbind(0))

    @staticmethod
    def backward(ctx, *gs):
        gs = [torch.zeros_like(gs[0] if gs[0] is not None else next(x for x in gs if x is not None))
              if g is None else g for g in gs]
        return (None, None) + tuple(_gather(ctx.ex, ctx.grp, gs))


class _UlyssesGather(torch.autograd.Function):
    """Tensors [B, N, H/S, D] (all rows, heads of member j) → [B, n_j, H, D]."""

    @staticmethod
    def forward(ctx, ex, grp, *ts):
        ctx.ex, ctx.grp = ex, grp
        return tuple(_gather(ex, grp, ts))

    @staticmethod
    def backward(ctx, *gs):
        gs = [torch.zeros_like(next(x for x in gs if x is not None)) if g is None else g for g in gs]
        S, j, base, splits = ctx.grp
        B, _, H, D = gs[0].shape
        rank, off, chunk = ulysses_tables(S, j, base, splits, B, H, D, gs[0].element_size(), len(gs), True)
        out = torch.empty(len(gs), B, sum(splits), H // S, D, dtype=gs[0].dtype, device=gs[0].device)
        _pull(ctx.ex, gs, out, rank, off, 1, chunk, False)
        return (None, None) + tuple(out.unbind(0))


def _gather(ex, grp, ts):
    S, j, base, splits = grp
    B, N, hs, D = ts[0].shape
    rank, off, chunk = ulysses_tables(S, j, base, splits, B, hs * S, D, ts[0].element_size(), len(ts), False)
    out = torch.empty(len(ts), B, splits[j], hs * S, D, dtype=ts[0].dtype, device=ts[0].device)
    _pull(ex, ts, out, rank, off, 1, chunk, False)
    return out.unbind(0)


def ulysses_group_of(spec: ParallelSpec, dense: bool) -> Tuple[int, int, int]:
    """(size, my index, first global SP rank) of this rank's Ulysses group: the ``full_sp``
    consecutive ranks in dense blocks, the ``ulysses`` consecutive ranks in sparse ones."""
    S = spec.full_sp if dense else spec.ulysses
    j = spec.rank % S
    return S, j, spec.rank - j


def p2p_ulysses_scatter(ex, grp, *ts):
    """Row shards → head shards for one or more tensors in one exchange (differentiable)."""
    return _UlyssesScatter.apply(ex, grp, *ts)


def p2p_ulysses_gather(ex, grp, *ts):
    """Head shards → row shards (differentiable)."""
    return _UlyssesGather.apply(ex, grp, *ts)
