"""Attach sequence parallelism to a model.

``build_sp_groups`` creates the process groups for a (dp, cfg, ssp, ulysses)
decomposition of the world (reference meshes: train_osp.py:121-161,
infer_osp.py:82-120; CFG-parallel is an addition of this framework) and
``attach_sp`` gives the model an :class:`SPRuntime` whose
:class:`~osp_next_b200.models.layout.ParallelSpec` drives every token layout.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch.distributed as dist

from ..models.layout import ParallelSpec
from .sp_state import sp_state


@dataclass
class SPRuntime:
    spec: ParallelSpec
    global_sp_group: object = None
    ulysses_group: object = None
    full_group: object = None
    skiparse_group: object = None
    p2p: object = None            # parallel.p2p.P2PExchange when the fused NVLink exchange is on


def _new_groups(world: int, size: int, stride: int = 1, block: int = None):
    """All groups of `size` ranks; returns the group containing this rank."""
    me = dist.get_rank()
    mine = None
    block = block or size * stride
    for base in range(0, world, block):
        for off in range(stride):
            ranks = [base + off + i * stride for i in range(size)]
            if max(ranks) >= world:
                continue
            g = dist.new_group(ranks)
            if me in ranks:
                mine = g
    return mine


def build_sp_groups(num_heads: int, skiparse_sp_size: int = 1, sp_size: int = 1, cfg_size: int = 1):
    """Rank layout (fastest varying first): ulysses, ssp, cfg, dp.

    Returns an :class:`SPRuntime` for this rank.  Every rank calls this with the
    same arguments (c10d group creation is collective).
    """
    world = dist.get_world_size() if dist.is_initialized() else 1
    gsp = skiparse_sp_size * sp_size
    if world % (gsp * cfg_size) != 0:
        raise ValueError(f"world {world} not divisible by ssp·ulysses·cfg = {gsp * cfg_size}")
    if world == 1 or not dist.is_initialized():
        return SPRuntime(ParallelSpec(1, 1, 1, 0))
    me = dist.get_rank()
    global_sp = _new_groups(world, gsp) if gsp > 1 else None
    ulysses = _new_groups(world, sp_size) if sp_size > 1 else None
    ssp = _new_groups(world, skiparse_sp_size, stride=sp_size, block=gsp) if skiparse_sp_size > 1 else None
    full = math.gcd(num_heads, gsp)
    full_group = _new_groups(world, full) if full > 1 else None
    cfg = _new_groups(world, cfg_size, stride=gsp, block=gsp * cfg_size) if cfg_size > 1 else None
    sp_state.reset(global_sp_group=global_sp, sp_group=ulysses, skiparse_sp_group=ssp,
                   full_sp_group=full_group, cfg_group=cfg)
    spec = ParallelSpec(ssp=skiparse_sp_size, ulysses=sp_size, full_sp=full, rank=me % gsp)
    return SPRuntime(spec, global_sp, ulysses, full_group, ssp)


def attach_sp(model, runtime: Optional[SPRuntime]):
    base = getattr(model, "base_model", None)
    target = model
    while hasattr(target, "module") and not hasattr(target, "block_kinds"):
        target = target.module
    if base is not None and hasattr(base, "model"):
        target = base.model
    target.parallel = runtime if (runtime is not None and runtime.spec.world > 1) else None
    return model


def enable_p2p_exchange(model, batch: int, grid, device, limit_s: float = 2.0):
    """Move the model's layout changes and Ulysses all-to-alls onto NVLink peer memory.

    Inference stores FFN-down rows straight into the owners' residual slots when every
    row has one owner (``full_sp == world``); every other exchange, and all of them under
    autograd, is a staged pull.  Slots are sized for the largest per-rank row count over
    the model's layouts, for ``batch`` samples of ``grid`` patches: fp32 residual rows,
    and for staging bf16 q, k and v together (the largest staged exchange).  ``limit_s``
    bounds each device barrier (a training step may wait on a slower rank for longer).
    """
    from ..models.layout import ParallelSpec, make_layout
    from .p2p import P2PExchange
    rt = getattr(model, "parallel", None)
    if rt is None or rt.spec.world == 1:
        return None
    P = model.sparse_ratio
    n_stride = 0
    for kind in set(model.block_kinds):
        for r in range(rt.spec.world):
            sp = ParallelSpec(rt.spec.ssp, rt.spec.ulysses, rt.spec.full_sp, r)
            n_stride = max(n_stride, make_layout(kind, tuple(grid), P, sp).n_local)
    # q, k, v (or their gradients) in bf16: 3 × 2 bytes per element; a Ulysses member's
    # share of the rows (Σ splits / size) never exceeds the largest n_local
    stage = 6 * batch * n_stride * model.dim + 64
    rt.p2p = P2PExchange(rt.global_sp_group, batch, n_stride, model.dim, device, stage_bytes=stage, limit_s=limit_s)
    return rt.p2p
