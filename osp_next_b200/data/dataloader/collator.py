"""Batch collators (reference: ospnext/data/dataloader/collator.py:4-21)."""
import torch

from ...utils.constant import PROMPT_IDS, PROMPT_MASK, VIDEO


class WanDataCollator:
    def __init__(self, *args, **kwargs):
        pass

    def __call__(self, batch):
        video = torch.stack([b[VIDEO] for b in batch]) if batch[0][VIDEO] is not None else None
        ids = torch.cat([b[PROMPT_IDS] for b in batch])
        mask = torch.cat([b[PROMPT_MASK] for b in batch]) if batch[0][PROMPT_MASK] is not None else None
        return {VIDEO: video, PROMPT_IDS: ids, PROMPT_MASK: mask}


class LatentCollator:
    def __init__(self, *args, **kwargs):
        pass

    def __call__(self, batch):
        return {k: torch.stack([b[k] for b in batch]) for k in batch[0]}
