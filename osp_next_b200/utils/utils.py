"""Small helpers (reference: ospnext/utils/utils.py:9-136).

The reference's NPU detection / `transfer_to_npu` is intentionally absent: this
framework targets sm_100a only.
"""
from collections import OrderedDict
import threading

import torch
import torch.distributed as dist

STR_DTYPE_TO_TORCH_DTYPE = {
    "float32": torch.float32, "fp32": torch.float32,
    "float16": torch.float16, "fp16": torch.float16,
    "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
}
TORCH_DTYPE_TO_STR_DTYPE = {v: k for k, v in STR_DTYPE_TO_TORCH_DTYPE.items() if len(k) > 4}


def to_dtype(d):
    if isinstance(d, torch.dtype):
        return d
    return STR_DTYPE_TO_TORCH_DTYPE[str(d)]


def safe_get_rank() -> int:
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def safe_get_world_size() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def contiguous(x):
    return x if x is None or x.is_contiguous() else x.contiguous()


def get_memory_allocated(device=None) -> float:
    """GiB currently allocated by the torch caching allocator on `device`."""
    if not torch.cuda.is_available():
        return 0.0
    return torch.cuda.memory_allocated(device) / 1024 ** 3


class SafeCacheManager:
    """Thread-safe bounded LRU cache (reference utils.py SafeCacheManager)."""

    def __init__(self, max_cache_size: int = 16):
        self.max_cache_size = max_cache_size
        self._d = OrderedDict()
        self._lock = threading.Lock()

    def is_exist(self, key) -> bool:
        with self._lock:
            return key in self._d

    def get(self, key):
        with self._lock:
            v = self._d.pop(key)
            self._d[key] = v
            return v

    def set(self, key, value) -> None:
        with self._lock:
            if key in self._d:
                self._d.pop(key)
            self._d[key] = value
            while len(self._d) > self.max_cache_size:
                self._d.popitem(last=False)

    def clear(self) -> None:
        with self._lock:
            self._d.clear()
