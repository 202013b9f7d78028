"""Process-group registry for sequence/CFG parallelism.

Same roles as the reference's singleton (ospnext/distributed/sp_state.py:5-113):
global SP group (all ranks sharing one sample), Ulysses group, Skiparse-SP group
and the dense-block ("full-blocks") group, plus a CFG group (cond/uncond split
across ranks) that the reference does not have.
"""
from __future__ import annotations

from typing import Optional

import torch.distributed as dist
from torch.distributed import ProcessGroup


class SequenceParallelState:
    def __init__(self):
        self.reset_counts = 0
        self._clear()

    def _clear(self):
        self.global_rank = 0
        self.global_sp_group: Optional[ProcessGroup] = None
        self.global_sp_rank = 0
        self.global_sp_size = 1
        self.sp_group: Optional[ProcessGroup] = None
        self.sp_rank = 0
        self.sp_size = 1
        self.skiparse_sp_group: Optional[ProcessGroup] = None
        self.skiparse_sp_rank = 0
        self.skiparse_sp_size = 1
        self.full_sp_group: Optional[ProcessGroup] = None
        self.full_sp_rank = 0
        self.full_sp_size = 1
        self.cfg_group: Optional[ProcessGroup] = None
        self.cfg_rank = 0
        self.cfg_size = 1
        self.is_initialized = False

    @staticmethod
    def _info(g):
        if g is None:
            return 0, 1
        return dist.get_rank(g), dist.get_world_size(g)

    def reset(self, global_sp_group=None, sp_group=None, skiparse_sp_group=None, full_sp_group=None, cfg_group=None):
        self.global_rank = dist.get_rank() if dist.is_initialized() else 0
        for name, g in (("global_sp", global_sp_group), ("sp", sp_group), ("skiparse_sp", skiparse_sp_group),
                        ("full_sp", full_sp_group), ("cfg", cfg_group)):
            if g is not None:
                r, s = self._info(g)
                setattr(self, f"{name}_group", g)
                setattr(self, f"{name}_rank", r)
                setattr(self, f"{name}_size", s)
        self.is_initialized = True
        self.reset_counts += 1

    def clear(self):
        self._clear()

    def get_sp_infos_with_type(self, sp_type: str):
        return {
            "sp": (self.sp_group, self.sp_rank, self.sp_size),
            "skiparse_sp": (self.skiparse_sp_group, self.skiparse_sp_rank, self.skiparse_sp_size),
            "full_blocks_sp": (self.full_sp_group, self.full_sp_rank, self.full_sp_size),
            "global_sp": (self.global_sp_group, self.global_sp_rank, self.global_sp_size),
        }[sp_type]


sp_state = SequenceParallelState()


def use_sequence_parallel() -> bool:
    return sp_state.is_initialized and sp_state.sp_size > 1


def use_skiparse_sequence_parallel() -> bool:
    return sp_state.is_initialized and sp_state.skiparse_sp_size > 1


def use_full_blocks_sequence_parallel() -> bool:
    return sp_state.is_initialized and sp_state.full_sp_size > 1
