"""Resumable distributed sampler (reference: ospnext/data/dataloader/sampler.py:12-126).

Shuffles with ``seed + epoch``, pads to a multiple of the world size, hands rank
``r`` every world-th index, and records how many indices it has yielded so a
resumed run continues mid-epoch.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch.utils.data import Sampler


class StatefulDistributedSampler(Sampler):
    def __init__(self, dataset, num_replicas=None, rank=None, shuffle=True, seed=0, drop_last=False):
        if num_replicas is None:
            num_replicas = dist.get_world_size() if dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank() if dist.is_initialized() else 0
        self.dataset = dataset
        self.num_replicas = num_replicas
        self.rank = rank
        self.shuffle = shuffle
        self.seed = seed
        self.drop_last = drop_last
        self.epoch = 0
        self.yielded = 0
        self.next_yielded = None
        n = len(dataset)
        if drop_last and n % num_replicas:
            self.num_samples = n // num_replicas
        else:
            self.num_samples = math.ceil(n / num_replicas)
        self.total_size = self.num_samples * num_replicas

    def _indices(self):
        n = len(self.dataset)
        if self.shuffle:
            g = torch.Generator()
            g.manual_seed(self.seed + self.epoch)
            idx = torch.randperm(n, generator=g).tolist()
        else:
            idx = list(range(n))
        if not self.drop_last:
            pad = self.total_size - len(idx)
            idx += (idx * math.ceil(pad / max(1, len(idx))))[:pad]
        else:
            idx = idx[: self.total_size]
        return idx[self.rank: self.total_size: self.num_replicas]

    def __iter__(self):
        if self.next_yielded is not None:
            self.yielded = self.next_yielded
            self.next_yielded = None
        idx = self._indices()
        for i in idx[self.yielded:]:
            self.yielded += 1
            yield i
        self.yielded = 0
        self.epoch += 1

    def __len__(self):
        return self.num_samples

    def set_epoch(self, epoch):
        self.epoch = epoch

    def state_dict(self):
        return {"yielded": self.yielded, "epoch": self.epoch, "seed": self.seed}

    def load_state_dict(self, sd):
        self.next_yielded = sd["yielded"]
        self.epoch = sd["epoch"]
        self.seed = sd.get("seed", self.seed)
