"""Loader for the in-tree sm_100a extension ``osp_next_b200/ops/_C.so``.

CUDA tensors always go through the extension.  If it is missing on a GPU box the
call raises (there is no silent PyTorch fallback on the GPU path); CPU tensors
use the PyTorch reference math in :mod:`osp_next_b200.ops.reference`.
"""
import importlib
import os

_EXT = None
_ERR = None
_LAUNCHES = [0]


class _Counted:
    """Proxy over the extension module that counts kernel-launching calls."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if name.startswith("get_"):
            return fn

        def call(*a, **k):
            _LAUNCHES[0] += 1
            return fn(*a, **k)
        return call


def launch_count() -> int:
    """Number of extension kernel calls made so far in this process."""
    return _LAUNCHES[0]


def ext():
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        import torch  # noqa: F401  (libtorch must be loaded before the extension)
        _EXT = _Counted(importlib.import_module("osp_next_b200.ops._C"))
    except ImportError as e:  # pragma: no cover - exercised only on misconfigured boxes
        _ERR = e
        raise RuntimeError(
            "osp_next_b200 CUDA extension (_C) is not built. Build it with "
            "`python -m osp_next_b200.ops.build` (nvcc, sm_100a)."
        ) from e
    return _EXT


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def so_path() -> str:
    return os.path.join(os.path.dirname(__file__), "_C.so")
