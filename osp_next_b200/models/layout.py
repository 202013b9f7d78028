"""Skiparse-2D token layouts as explicit index maps.

The reference expresses Skiparse with einops permutations on a zero-padded grid
(ospnext/modules/skiparse_func.py:18-55, osp_next.py:146-283) and shards the
permuted batch dimension across SSP ranks (osp_next.py:174-189).  Here the same
semantics are expressed as *index maps over the natural token order*:

* token ``n`` of a ``T×H×W`` patch grid sits at ``(t, h, w)`` with
  ``n = (t·H + h)·W + w`` (``b c f h w -> b (f h w) c`` in osp_next.py:1341).
* a Token block (sparse ratio ``P``) attends inside the group
  ``gid = (h mod P)·P + (w mod P)``  — a stride-``P`` dilated grid.
* a Group block attends inside ``gid = ⌊(h mod P²)/P⌋·P + ⌊(w mod P²)/P⌋`` —
  ``P×P`` blocks repeating every ``P²`` rows/columns.
* inside a group, tokens keep natural order, which is exactly the order the
  reference's einops patterns produce.

Padding.  The reference pads ``H, W`` to multiples of ``P²`` and masks padded keys
(osp_next.py:221-260, 467-548).  Padded tokens never influence real tokens there
(their keys are masked, their queries are dropped at the skiparse→full boundary),
so this framework never materialises them: groups simply hold the real tokens
they contain and may differ in length (variable-length attention segments).
Every real token keeps its true ``(t, h, w)`` for RoPE, as in the reference.

Sequence parallelism.  With ``S`` SSP ranks each rank owns ``G = P²/S`` whole
groups (``gid ∈ [r·G, (r+1)·G)``, the reference's ``narrow`` of the ``(p q b)``
batch dim).  Dense blocks split the natural order into contiguous chunks
(Ulysses; the reference's "full-blocks SP", osp_next.py:1185, 1263-1331).  The
residual stream on a rank is always the ordered list of tokens the rank owns in
the current block's layout; moving between two layouts is a *redistribution*
(:class:`Redistribution`): a permutation on one GPU, an all-to-all across ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache
from typing import List, Optional, Sequence, Tuple

import torch

FULL = "full"
TOKEN = "token"
GROUP = "group"


def block_schedule(num_layers: int, skiparse_model_type: str, num_full_blocks: int) -> Tuple[List[str], List[int]]:
    """Per-block kind list and the dense block indices.

    Mirrors osp_next.py:1108-1161: dense blocks are the first and last
    ``F/2`` blocks ("dual_end"); other blocks alternate Token (even index) /
    Group (odd index).  ``skiparse_model_type == "full"`` makes every block dense.
    """
    if skiparse_model_type == "full":
        return [FULL] * num_layers, list(range(num_layers))
    if not (num_layers % 2 == 0 and num_full_blocks % 2 == 0 and num_full_blocks <= num_layers // 2):
        raise ValueError("num_full_blocks should be divisible by 2 and <= num_layers // 2")
    if num_full_blocks == 0:
        full = []
    elif skiparse_model_type == "dual_end":
        if num_full_blocks % 4 != 0:
            raise ValueError("num_full_blocks should be divisible by 4")
        start = num_full_blocks // 2
        end = num_layers - num_full_blocks // 2 - 1
        if not start < end:
            raise ValueError("skiparse_start_index should be less than skiparse_end_index")
        full = list(range(0, start)) + list(range(end + 1, num_layers))
    else:
        raise ValueError(f"Unsupported skiparse model type: {skiparse_model_type}")
    kinds = []
    for i in range(num_layers):
        if i in full:
            kinds.append(FULL)
        elif i % 2 == 0:
            kinds.append(TOKEN)
        else:
            kinds.append(GROUP)
    return kinds, full


def group_ids(kind: str, grid: Sequence[int], P: int) -> torch.Tensor:
    """Group id of every token in natural order (int64 [T·H·W])."""
    T, H, W = grid
    h = torch.arange(H).view(1, H, 1).expand(T, H, W)
    w = torch.arange(W).view(1, 1, W).expand(T, H, W)
    if kind == FULL or P == 1:
        g = torch.zeros(T, H, W, dtype=torch.long)
    elif kind == TOKEN:
        g = (h % P) * P + (w % P)
    elif kind == GROUP:
        P2 = P * P
        g = ((h % P2) // P) * P + ((w % P2) // P)
    else:
        raise ValueError(kind)
    return g.reshape(-1).contiguous()


def num_groups(kind: str, P: int) -> int:
    return 1 if (kind == FULL or P == 1) else P * P


@dataclass(frozen=True)
class ParallelSpec:
    """How one sample's tokens are spread over ranks.

    ``ssp``: Skiparse-SP degree (divides ``P²``); ``ulysses``: head-split degree
    applied inside sparse blocks; dense blocks use Ulysses over
    ``full_sp = gcd(heads, ssp·ulysses)`` ranks (osp_next.py:1185 / train_osp.py:235-246).
    """
    ssp: int = 1
    ulysses: int = 1
    full_sp: int = 1
    rank: int = 0          # rank inside the global SP group (ssp-major, ulysses-minor)

    @property
    def world(self) -> int:
        return self.ssp * self.ulysses

    @property
    def ssp_rank(self) -> int:
        return self.rank // self.ulysses

    @property
    def ulysses_rank(self) -> int:
        return self.rank % self.ulysses

    @property
    def full_rank(self) -> int:
        return self.rank % self.full_sp


def _chunk_bounds(n: int, parts: int) -> List[int]:
    """Split ``n`` rows into ``parts`` near-equal contiguous chunks (torch.chunk rule)."""
    size = -(-n // parts)
    b = [min(i * size, n) for i in range(parts + 1)]
    return b


@dataclass
class TokenLayout:
    """Tokens one rank holds for one block kind, plus attention segments.

    ``tokens``  int64 [n_local]: natural indices of the rows this rank holds
                (residual-stream order).
    ``attn_tokens`` int64 [n_attn]: natural indices of the rows attention sees
                after the head all-to-all (== ``tokens`` without Ulysses).
    ``seg``     int32 [n_seg+1]: attention segment offsets into ``attn_tokens``.
    ``a2a_splits``  rows each Ulysses peer contributes to ``attn_tokens``
                (None without Ulysses).
    """
    kind: str
    tokens: torch.Tensor
    attn_tokens: torch.Tensor
    seg: torch.Tensor
    a2a_splits: Optional[List[int]]
    a2a_group_size: int

    @property
    def n_local(self) -> int:
        return int(self.tokens.numel())

    @property
    def max_seg_len(self) -> int:
        s = self.seg
        return int((s[1:] - s[:-1]).max().item()) if s.numel() > 1 else 0


def _full_owner(n_tokens: int, spec: ParallelSpec) -> torch.Tensor:
    """Owner (rank in global SP group) of each natural token in a dense block.

    Dense blocks use Ulysses over ``full_sp`` ranks; ranks ``r`` and
    ``r + full_sp`` … hold replicas of the same chunk (the reference's gcd rule).
    Only the first replica is the *owner* used as the source of redistributions.
    """
    b = _chunk_bounds(n_tokens, spec.full_sp)
    owner = torch.empty(n_tokens, dtype=torch.long)
    for i in range(spec.full_sp):
        owner[b[i]:b[i + 1]] = i
    return owner


@lru_cache(maxsize=64)
def make_layout(kind: str, grid: Tuple[int, int, int], P: int, spec: ParallelSpec) -> TokenLayout:
    T, H, W = grid
    N = T * H * W
    if kind == FULL or P == 1:
        F = spec.full_sp
        b = _chunk_bounds(N, F)
        fr = spec.full_rank
        tokens = torch.arange(b[fr], b[fr + 1], dtype=torch.long)
        attn_tokens = torch.arange(N, dtype=torch.long)
        seg = torch.tensor([0, N], dtype=torch.int32)
        splits = [b[i + 1] - b[i] for i in range(F)] if F > 1 else None
        return TokenLayout(kind, tokens, attn_tokens if F > 1 else tokens, seg, splits, F)

    G_total = P * P
    if G_total % spec.ssp != 0:
        raise ValueError(f"skiparse_sp_size={spec.ssp} must divide P²={G_total}")
    G = G_total // spec.ssp
    gid = group_ids(kind, grid, P)
    own = []
    seg = [0]
    for g in range(spec.ssp_rank * G, (spec.ssp_rank + 1) * G):
        idx = torch.nonzero(gid == g, as_tuple=False).flatten()
        own.append(idx)
        seg.append(seg[-1] + idx.numel())
    ssp_tokens = torch.cat(own)
    seg_t = torch.tensor(seg, dtype=torch.int32)
    if spec.ulysses == 1:
        return TokenLayout(kind, ssp_tokens, ssp_tokens, seg_t, None, 1)
    b = _chunk_bounds(ssp_tokens.numel(), spec.ulysses)
    ur = spec.ulysses_rank
    tokens = ssp_tokens[b[ur]:b[ur + 1]]
    splits = [b[i + 1] - b[i] for i in range(spec.ulysses)]
    return TokenLayout(kind, tokens, ssp_tokens, seg_t, splits, spec.ulysses)


def owner_map(kind: str, grid: Tuple[int, int, int], P: int, spec: ParallelSpec) -> Tuple[torch.Tensor, torch.Tensor]:
    """For every natural token: owning rank (global SP rank) and row on that rank."""
    T, H, W = grid
    N = T * H * W
    owner = torch.full((N,), -1, dtype=torch.long)
    row = torch.full((N,), -1, dtype=torch.long)
    if kind == FULL or P == 1:
        ranks = range(spec.full_sp)   # replicas beyond full_sp hold copies; owners are 0..F-1
    else:
        ranks = range(spec.world)
    for r in ranks:
        lay = make_layout(kind, grid, P, ParallelSpec(spec.ssp, spec.ulysses, spec.full_sp, r))
        owner[lay.tokens] = r
        row[lay.tokens] = torch.arange(lay.n_local)
    return owner, row


@dataclass
class Redistribution:
    """Move residual-stream rows from layout A to layout B (one rank's view).

    Single rank: ``x_B = x_A[:, gather]``.
    Multi rank: rows ``send_rows`` (grouped by destination, ``send_counts``) go
    out; received rows (grouped by source, ``recv_counts``) land at
    ``recv_rows`` of layout B.  ``dest_rank``/``dest_row`` give, for every local
    row of A, where it lives in B: the form a fused GEMM epilogue uses to store
    straight into the destination buffer.
    """
    gather: Optional[torch.Tensor]
    send_rows: Optional[torch.Tensor]
    send_counts: Optional[List[int]]
    recv_rows: Optional[torch.Tensor]
    recv_counts: Optional[List[int]]
    dest_rank: torch.Tensor
    dest_row: torch.Tensor
    n_out: int
    identity: bool


@lru_cache(maxsize=64)
def make_redistribution(kind_a: str, kind_b: str, grid: Tuple[int, int, int], P: int,
                        spec: ParallelSpec) -> Redistribution:
    la = make_layout(kind_a, grid, P, spec)
    lb = make_layout(kind_b, grid, P, spec)
    n_out = lb.n_local
    if spec.world == 1:
        N = grid[0] * grid[1] * grid[2]
        pos_a = torch.full((N,), -1, dtype=torch.long)
        pos_a[la.tokens] = torch.arange(la.n_local)
        gather = pos_a[lb.tokens]
        pos_b = torch.full((N,), -1, dtype=torch.long)
        pos_b[lb.tokens] = torch.arange(lb.n_local)
        dest_row = pos_b[la.tokens]
        ident = bool(torch.equal(gather, torch.arange(n_out)))
        return Redistribution(gather, None, None, None, None,
                              torch.zeros(la.n_local, dtype=torch.long), dest_row, n_out, ident)
    own_b, row_b = owner_map(kind_b, grid, P, spec)
    own_a, _ = owner_map(kind_a, grid, P, spec)
    # source rows: the tokens this rank *owns* in layout A (replicas don't send)
    my_a = la.tokens
    i_own = (own_a[my_a] == spec.rank)
    dest_rank_all = own_b[my_a]
    dest_row_all = row_b[my_a]
    # every destination replica of a dense chunk needs a copy: dense layout B
    # replicas r + k·full_sp also receive; represent those as extra sends.
    dests = []
    rows = []
    n_rep = spec.world // spec.full_sp if (kind_b == FULL or P == 1) else 1
    for k in range(n_rep):
        dr = dest_rank_all + k * spec.full_sp
        dests.append(torch.where(i_own, dr, torch.full_like(dr, -1)))
        rows.append(torch.arange(la.n_local))
    dest_all = torch.cat(dests)
    row_src = torch.cat(rows)
    send_rows, send_counts = [], []
    for r in range(spec.world):
        m = (dest_all == r)
        srcs = row_src[m]
        # order by destination row so the receiver can place data without metadata
        order = torch.argsort(dest_row_all[srcs])
        send_rows.append(srcs[order])
        send_counts.append(int(m.sum()))
    # receive side: tokens of my B layout, grouped by their A owner, ordered by B row
    my_b = lb.tokens
    src_of = own_a[my_b]
    recv_rows, recv_counts = [], []
    for r in range(spec.world):
        m = torch.nonzero(src_of == r, as_tuple=False).flatten()
        recv_rows.append(m)   # already sorted by B row
        recv_counts.append(int(m.numel()))
    return Redistribution(None, torch.cat(send_rows), send_counts, torch.cat(recv_rows), recv_counts,
                          dest_rank_all, dest_row_all, n_out, False)


def token_positions(tokens: torch.Tensor, grid: Sequence[int]) -> torch.Tensor:
    """(t, h, w) int32 [n, 3] of natural token indices."""
    T, H, W = grid
    t = tokens // (H * W)
    h = (tokens // W) % H
    w = tokens % W
    return torch.stack([t, h, w], dim=1).to(torch.int32)
