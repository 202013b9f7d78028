"""Skiparse index maps vs the reference's einops layouts, and redistribution maps."""
import pytest
import torch
from einops import rearrange

from osp_next_b200.models.layout import (FULL, GROUP, TOKEN, ParallelSpec, block_schedule, group_ids, make_layout,
                                         make_redistribution)


def _ref_token_groups(T, H, W, P):
    idx = torch.arange(T * H * W).view(1, T * H * W, 1)
    g = rearrange(idx, 'b (t h p w q) c -> (p q b) (t h w) c', p=P, q=P, h=H // P, w=W // P)
    return [g[i, :, 0] for i in range(P * P)]


def _ref_group_groups(T, H, W, P):
    idx = torch.arange(T * H * W).view(1, T * H * W, 1)
    g = rearrange(idx, 'b (txh p1 p2 w q1 q2) c -> (p1 q1 b) (txh p2 w q2) c', p1=P, q1=P, p2=P, q2=P,
                  w=W // (P * P))
    return [g[i, :, 0] for i in range(P * P)]


@pytest.mark.parametrize("T,H,W", [(3, 8, 12), (2, 16, 8)])
def test_token_and_group_layouts_match_einops(T, H, W):
    P = 2
    for kind, ref in ((TOKEN, _ref_token_groups(T, H, W, P)), (GROUP, _ref_group_groups(T, H, W, P))):
        lay = make_layout(kind, (T, H, W), P, ParallelSpec())
        seg = lay.seg.tolist()
        for g in range(P * P):
            assert torch.equal(lay.tokens[seg[g]:seg[g + 1]], ref[g])


def test_padded_grid_groups_drop_padding():
    T, H, W, P = 2, 9, 11, 2
    gid = group_ids(TOKEN, (T, H, W), P)
    lay = make_layout(TOKEN, (T, H, W), P, ParallelSpec())
    assert lay.n_local == T * H * W
    assert sorted(lay.tokens.tolist()) == list(range(T * H * W))
    for g in range(4):
        s = lay.seg.tolist()
        assert bool((gid[lay.tokens[s[g]:s[g + 1]]] == g).all())


def test_block_schedule():
    kinds, full = block_schedule(40, "dual_end", 8)
    assert full == [0, 1, 2, 3, 36, 37, 38, 39]
    assert kinds[4] == TOKEN and kinds[5] == GROUP and kinds[35] == GROUP
    with pytest.raises(ValueError):
        block_schedule(2, "dual_end", 4)


@pytest.mark.parametrize("ssp", [2, 4])
def test_ssp_partition_and_redistribution(ssp):
    grid, P = (3, 8, 12), 2
    N = 3 * 8 * 12
    for kind in (TOKEN, GROUP):
        seen = torch.cat([make_layout(kind, grid, P, ParallelSpec(ssp, 1, 1, r)).tokens for r in range(ssp)])
        assert sorted(seen.tolist()) == list(range(N))
    # simulate the all-to-all with the per-rank plans
    x = {r: make_layout(TOKEN, grid, P, ParallelSpec(ssp, 1, 1, r)).tokens.float() for r in range(ssp)}
    plans = {r: make_redistribution(TOKEN, GROUP, grid, P, ParallelSpec(ssp, 1, 1, r)) for r in range(ssp)}
    for dst in range(ssp):
        pl = plans[dst]
        out = torch.full((pl.n_out,), -1.0)
        recv = []
        for src in range(ssp):
            ps = plans[src]
            off = sum(ps.send_counts[:dst])
            recv.append(x[src][ps.send_rows[off:off + ps.send_counts[dst]]])
        out[pl.recv_rows] = torch.cat(recv)
        assert torch.equal(out, make_layout(GROUP, grid, P, ParallelSpec(ssp, 1, 1, dst)).tokens.float())


def test_single_gpu_dest_rows_invert_gather():
    grid, P = (2, 8, 8), 2
    rd = make_redistribution(TOKEN, GROUP, grid, P, ParallelSpec())
    src = make_layout(TOKEN, grid, P, ParallelSpec()).tokens
    dst = torch.empty_like(src)
    dst[rd.dest_row] = src
    assert torch.equal(dst, make_layout(GROUP, grid, P, ParallelSpec()).tokens)
    assert torch.equal(src[rd.gather], dst)
