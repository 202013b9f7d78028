"""Fused SSP exchange over NVLink: peer buffers + epilogue stores + bounded barrier.

At every layout change between blocks (Token↔Group between sparse blocks, and the
dense↔sparse boundaries) the residual stream must move to the ranks that own each
token in the next layout.  The reference does a local permute, one NCCL
``all_to_all_single`` and another permute (ospnext/modules/skiparse_func.py:58-93).
Here the block's last GEMM (FFN-down + gated residual) stores every output row
directly into the owner rank's buffer (``ops.linear_gated_residual_p2p``), so the
exchange overlaps the GEMM tile by tile and no permute or copy pass exists; a
bounded flag barrier (``p2p_barrier``) then orders the stores before the next
block reads its buffer.

Buffers: two residual buffers per rank (ping-pong: block i reads A and writes the
peers' B), ``[B, n_stride, C]`` fp32 with one common row stride, allocated with
``cudaMalloc`` and shared through CUDA IPC handles (plain loads/stores over
NVLink, no multicast object).  Flags: one int per peer, monotonically increasing
epochs, so no reset is needed between steps.

A second ring of two staging slots serves the exchanges whose result must outlive the
next one (training, where autograd keeps it) and the Ulysses all-to-all: each rank copies
its rows into a staging slot, one barrier orders the copies, and every rank pulls the
chunks it owns into a fresh tensor (:mod:`osp_next_b200.parallel.p2p_collectives`).  Every
exchange on a slot ring is write → barrier → read, and a slot is written again only two
exchanges later, after a barrier that every rank reaches only once its reads of that slot
are done; so two slots per ring suffice.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops


class P2PExchange:
    """``batch × n_stride × channels`` fp32 residual slots (ring of two, fused GEMM-epilogue
    stores) and ``stage_bytes`` staging slots (ring of two, staged pulls) on every rank of
    ``group``, mapped by every peer; ``limit_s`` bounds each device barrier."""

    def __init__(self, group, batch: int, n_stride: int, channels: int, device, stage_bytes: int = 0,
                 limit_s: float = 2.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.batch, self.n_stride, self.channels = batch, n_stride, channels
        self.device = torch.device(device)
        self.limit_s = float(limit_s)
        ext = ops.ext()
        nbytes = batch * n_stride * channels * 4
        self.stage_bytes = int(stage_bytes) or nbytes
        sizes = [nbytes, nbytes, 4 * max(1, self.world), self.stage_bytes, self.stage_bytes]
        self._own: List[int] = []
        self._opened: List[int] = []
        handles = []
        for nb in sizes:
            ptr, h = ext.p2p_alloc(nb)
            self._own.append(ptr)
            handles.append(h)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=self.group)
        tables = [[0] * self.world for _ in sizes]
        for r in range(self.world):
            for k in range(len(sizes)):
                if r == self.rank:
                    tables[k][r] = self._own[k]
                else:
                    p = ext.p2p_open(gathered[r][k])
                    self._opened.append(p)
                    tables[k][r] = p
        self.data_ptrs = [torch.tensor(tables[k], dtype=torch.int64, device=self.device) for k in range(2)]
        self.flag_ptrs = torch.tensor(tables[2], dtype=torch.int64, device=self.device)
        self.stage_ptrs = [torch.tensor(tables[k], dtype=torch.int64, device=self.device) for k in (3, 4)]
        self._stage_own = [self._own[3], self._own[4]]
        self.epoch = 0
        self.cur = 0
        self.stage_cur = 0
        dist.barrier(group=self.group)

    def target(self):
        """Pointer table of the buffer the next store goes to (alternates every exchange)."""
        return self.data_ptrs[self.cur]

    def barrier(self, limit_s: Optional[float] = None):
        self.epoch += 1
        ops.ext().p2p_barrier(self.flag_ptrs, self.rank, self.world, self.epoch,
                              self.limit_s if limit_s is None else float(limit_s))

    def stage(self, tensors) -> torch.Tensor:
        """Copy ``tensors`` (contiguous, back to back, each start 16-byte aligned) into this
        rank's next staging slot, then barrier; returns the peers' pointer table of that slot
        (the pull that follows reads it)."""
        k = self.stage_cur
        self.stage_cur ^= 1
        off = 0
        for t in tensors:
            nb = t.numel() * t.element_size()
            if off + nb > self.stage_bytes:
                raise ValueError(f"P2PExchange.stage: {off + nb} bytes exceed the {self.stage_bytes}-byte slot")
            view = ops.ext().p2p_view(self._stage_own[k] + off, [t.numel()], t.dtype, self.device.index)
            view.copy_(t.reshape(-1))
            off += (nb + 15) // 16 * 16
        self.barrier()
        return self.stage_ptrs[k]

    def take(self, n_local: int) -> torch.Tensor:
        """Local view [B, n_local, C] of the buffer just written by the peers; flips ping-pong."""
        v = ops.ext().p2p_view(self._own[self.cur], [self.batch, self.n_stride, self.channels], torch.float32,
                               self.device.index)
        self.cur ^= 1
        return v[:, :n_local]

    def close(self):
        ext = ops.ext()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            ext.p2p_close(p)
        dist.barrier(group=self.group)
        for p in self._own:
            ext.p2p_free(p)
        self._opened, self._own = [], []
