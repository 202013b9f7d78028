"""Stateful dataset base: Python/NumPy/torch RNG captured for exact resume
(reference: ospnext/data/datasets/base_dataset.py:9-24)."""
import random

import numpy as np
import torch
from torch.utils.data import Dataset


class BaseDataset(Dataset):
    def state_dict(self):
        return {"rng_random": random.getstate(), "rng_numpy": np.random.get_state(),
                "rng_torch": torch.get_rng_state()}

    def load_state_dict(self, sd):
        random.setstate(sd["rng_random"])
        np.random.set_state(sd["rng_numpy"])
        torch.set_rng_state(sd["rng_torch"])
