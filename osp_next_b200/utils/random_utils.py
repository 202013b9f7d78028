"""Seeding and determinism (reference: ospnext/utils/random_utils.py:10-53).

`set_seed(seed, device_specific=True)` offsets the seed by the global rank so
that data-parallel ranks draw different noise, exactly like the reference.
"""
import os
import random

import numpy as np
import torch
import torch.distributed as dist


def set_seed(seed: int, device_specific: bool = False, process_group=None) -> int:
    if device_specific:
        rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        seed = seed + rank
    random.seed(seed)
    np.random.seed(seed % (2 ** 32))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    return seed


def set_deterministic(enabled: bool = True) -> None:
    """Deterministic algorithms for torch ops; our own kernels are deterministic by
    construction (fixed reduction order, no atomics in the numerics path)."""
    torch.use_deterministic_algorithms(enabled, warn_only=True)
    torch.backends.cudnn.deterministic = enabled
    torch.backends.cudnn.benchmark = not enabled
    if enabled:
        os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")


def get_rng_state() -> dict:
    state = {
        "python": random.getstate(),
        "numpy": np.random.get_state(),
        "torch": torch.get_rng_state(),
    }
    if torch.cuda.is_available():
        state["cuda"] = torch.cuda.get_rng_state_all()
    return state


def set_rng_state(state: dict) -> None:
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"])
    if "cuda" in state and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(state["cuda"])
