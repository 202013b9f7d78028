"""Encoder-output sharing inside an SP group (reference: ospnext/utils/encoder_cache.py:5-39).

With ``global_sp`` ranks cooperating on one sample, each rank encodes (VAE + T5)
a *different* sample once every ``global_sp`` steps; then ranks take turns
broadcasting their cached (latent, text) to the group, so no encoder work is
duplicated inside the group.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist

from ..parallel.dist_utils import broadcast_tensor_list


class EncoderCacheManager:
    def __init__(self, sp_group=None):
        self.sp_group = sp_group
        self.sp_size = dist.get_world_size(sp_group) if (sp_group is not None and dist.is_initialized()) else 1
        self.sp_rank = dist.get_rank(sp_group) if (sp_group is not None and dist.is_initialized()) else 0
        self.cache: Optional[List[torch.Tensor]] = None
        self.step = 0

    def need_encode(self) -> bool:
        return self.step % self.sp_size == 0

    def set_cache(self, tensors: List[torch.Tensor]):
        self.cache = tensors

    def __call__(self) -> List[torch.Tensor]:
        """The tensors of this step: the owner (rank ``step % sp``) broadcasts its cache."""
        owner = self.step % self.sp_size
        self.step += 1
        if self.sp_size == 1:
            return self.cache
        src = dist.get_global_rank(self.sp_group, owner)
        return broadcast_tensor_list(self.cache if self.sp_rank == owner else None, src=src, group=self.sp_group,
                                     device=self.cache[0].device if self.cache else None)
