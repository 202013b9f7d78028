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
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops


class P2PExchange:
    def __init__(self, group, batch: int, n_stride: int, channels: int, device):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.batch, self.n_stride, self.channels = batch, n_stride, channels
        self.device = torch.device(device)
        ext = ops.ext()
        nbytes = batch * n_stride * channels * 4
        self._own: List[int] = []
        self._opened: List[int] = []
        handles = []
        for _ in range(2):
            ptr, h = ext.p2p_alloc(nbytes)
            self._own.append(ptr)
            handles.append(h)
        fptr, fh = ext.p2p_alloc(4 * max(1, self.world))
        self._own.append(fptr)
        handles.append(fh)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=self.group)
        tables = [[0] * self.world for _ in range(3)]
        for r in range(self.world):
            for k in range(3):
                if r == self.rank:
                    tables[k][r] = self._own[k]
                else:
                    p = ext.p2p_open(gathered[r][k])
                    self._opened.append(p)
                    tables[k][r] = p
        self.data_ptrs = [torch.tensor(tables[k], dtype=torch.int64, device=self.device) for k in range(2)]
        self.flag_ptrs = torch.tensor(tables[2], dtype=torch.int64, device=self.device)
        self.epoch = 0
        self.cur = 0
        dist.barrier(group=self.group)

    def target(self):
        """Pointer table of the buffer the next store goes to (alternates every exchange)."""
        return self.data_ptrs[self.cur]

    def barrier(self, limit_s: float = 2.0):
        self.epoch += 1
        ops.ext().p2p_barrier(self.flag_ptrs, self.rank, self.world, self.epoch, float(limit_s))

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
