"""Pull tables of the NVLink SSP exchange and Ulysses all-to-all, replayed on the CPU.

Every rank's staging slot is built the way ``P2PExchange.stage`` writes it, the table is
replayed with ``emulate_pull``, and the result must equal the exchange's definition: rows
of the next layout (forward), the owner's sum of every holder's gradient with zeros for
replica rows (backward), and the Ulysses head/row re-sharding.
"""
import pytest
import torch

from osp_next_b200.models.layout import FULL, GROUP, TOKEN, ParallelSpec, make_layout, owner_map
from osp_next_b200.parallel.p2p_collectives import (emulate_pull, redistribute_tables, stage_bytes,
                                                    ulysses_group_of, ulysses_tables)

GRID = (3, 6, 10)          # T, H, W patches (odd sizes: uneven chunks and padded groups)
P = 2

SPECS = [(2, 1, 2), (4, 1, 4), (4, 1, 2), (2, 2, 2), (2, 2, 4)]     # (ssp, ulysses, full_sp)
PAIRS = [(FULL, TOKEN), (TOKEN, GROUP), (GROUP, TOKEN), (GROUP, FULL), (TOKEN, FULL)]


def _specs(ssp, ul, full):
    return [ParallelSpec(ssp, ul, full, r) for r in range(ssp * ul)]


@pytest.mark.parametrize("ssp,ul,full", SPECS)
@pytest.mark.parametrize("ka,kb", PAIRS)
def test_redistribute_tables_forward_and_backward(ssp, ul, full, ka, kb):
    Bn, C = 2, 8
    N = GRID[0] * GRID[1] * GRID[2]
    specs = _specs(ssp, ul, full)
    g = torch.Generator().manual_seed(0)
    X = torch.randn(Bn, N, C, generator=g)
    xs = [X[:, make_layout(ka, GRID, P, s).tokens] for s in specs]
    stages = [stage_bytes([x]) for x in xs]
    # forward: every rank ends with its rows of layout B
    outs = []
    for s in specs:
        n_in, n_out, fr, fo, br, bo, R = redistribute_tables(ka, kb, GRID, P, s, Bn, C, 4, 4)
        out = torch.empty(Bn, n_out, C)
        emulate_pull(stages, fr, fo, 1, C * 4, False, out)
        assert torch.equal(out, X[:, make_layout(kb, GRID, P, s).tokens])
        outs.append(out)
    # backward: gradients of every holder of a B row summed at the A owner
    gs = [torch.randn(o.shape, generator=g) for o in outs]
    G = torch.zeros(Bn, N, C)
    for s, gr in zip(specs, gs):
        G[:, make_layout(kb, GRID, P, s).tokens] += gr
    gstages = [stage_bytes([x]) for x in gs]
    own_a, _ = owner_map(ka, GRID, P, specs[0])
    for s in specs:
        n_in, n_out, fr, fo, br, bo, R = redistribute_tables(ka, kb, GRID, P, s, Bn, C, 4, 4)
        dx = torch.empty(Bn, n_in, C)
        emulate_pull(gstages, br, bo, R, C * 4, R > 1, dx)
        tok = make_layout(ka, GRID, P, s).tokens
        exp = torch.where((own_a[tok] == s.rank)[None, :, None], G[:, tok], torch.zeros(()))
        torch.testing.assert_close(dx, exp)


@pytest.mark.parametrize("ssp,ul,full", [(2, 2, 2), (1, 4, 4), (4, 1, 4), (2, 2, 4)])
@pytest.mark.parametrize("kind", [FULL, TOKEN])
def test_ulysses_tables_scatter_and_gather(ssp, ul, full, kind):
    Bn, H, D = 2, 8, 8
    specs = _specs(ssp, ul, full)
    lays = [make_layout(kind, GRID, P, s) for s in specs]
    if lays[0].a2a_splits is None:
        pytest.skip("no Ulysses group in this layout")
    dense = kind == FULL
    g = torch.Generator().manual_seed(1)
    q = [torch.randn(Bn, l.n_local, H, D, generator=g).to(torch.bfloat16) for l in lays]
    k = [torch.randn_like(x, dtype=torch.float32).to(torch.bfloat16) for x in q]
    stages = [stage_bytes([a, b]) for a, b in zip(q, k)]
    heads = []
    for s, lay in zip(specs, lays):
        S, j, base = ulysses_group_of(s, dense)
        splits = tuple(lay.a2a_splits)
        rank, off, chunk = ulysses_tables(S, j, base, splits, Bn, H, D, 2, 2, True)
        out = torch.empty(2, Bn, sum(splits), H // S, D, dtype=torch.bfloat16)
        emulate_pull(stages, rank, off, 1, chunk, False, out)
        hs = H // S
        members = range(base, base + S)
        exp_q = torch.cat([q[m][:, :, j * hs:(j + 1) * hs] for m in members], 1)
        exp_k = torch.cat([k[m][:, :, j * hs:(j + 1) * hs] for m in members], 1)
        assert torch.equal(out[0], exp_q) and torch.equal(out[1], exp_k)
        heads.append(out[0].clone())
    # gather is the inverse: heads → rows gives back each rank's q
    hstages = [stage_bytes([h]) for h in heads]
    for s, lay in zip(specs, lays):
        S, j, base = ulysses_group_of(s, dense)
        splits = tuple(lay.a2a_splits)
        rank, off, chunk = ulysses_tables(S, j, base, splits, Bn, H, D, 2, 1, False)
        out = torch.empty(1, Bn, splits[j], H, D, dtype=torch.bfloat16)
        emulate_pull(hstages, rank, off, 1, chunk, False, out)
        assert torch.equal(out[0], q[s.rank])
