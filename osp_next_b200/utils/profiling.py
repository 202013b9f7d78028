"""Trainer profiling: a torch.profiler window and NVTX ranges (reference: train/train_osp.py:469-491).

``profiling`` in a trainer config is either ``false``, ``true`` (the reference's window:
iterations 5 and 6 are traced, then the run stops) or a dict
``{start: 5, steps: 2, exit_after: true}``.  Each traced iteration's forward and backward
run under ``torch.profiler.profile`` (CPU + CUDA activities, stacks and module names) and
the chrome trace is written to ``output_dir/trace_rank{rank}_{iteration:09d}.json``.

NVTX ranges (``nvtx: true`` in the config or ``OSP_NVTX=1`` in the environment) mark the
trainer phases and each DiT block, for Nsight Systems timelines; disabled they cost one
flag check.
"""
from __future__ import annotations

import contextlib
import os
from typing import Optional

import torch

_NVTX = [os.environ.get("OSP_NVTX", "0") == "1"]


def enable_nvtx(on: bool = True) -> None:
    _NVTX[0] = bool(on)


def nvtx_enabled() -> bool:
    return _NVTX[0]


@contextlib.contextmanager
def nvtx_range(name: str):
    if not _NVTX[0] or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


class ProfileWindow:
    """Decides per iteration whether to trace, and writes the trace."""

    def __init__(self, spec, output_dir: str, rank: int):
        if spec is True:
            spec = {"start": 5, "steps": 2, "exit_after": True}
        self.spec = dict(spec) if isinstance(spec, dict) else None
        self.output_dir = output_dir
        self.rank = rank

    @property
    def enabled(self) -> bool:
        return self.spec is not None

    def active(self, iteration: int) -> bool:
        if self.spec is None:
            return False
        s = int(self.spec.get("start", 5))
        return s <= iteration < s + int(self.spec.get("steps", 2))

    def finished(self, iteration: int) -> bool:
        """True after the last traced iteration when the run should stop (reference behaviour)."""
        if self.spec is None or not self.spec.get("exit_after", True):
            return False
        return iteration >= int(self.spec.get("start", 5)) + int(self.spec.get("steps", 2))

    @contextlib.contextmanager
    def __call__(self, iteration: int):
        if not self.active(iteration):
            yield None
            return
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        prof = torch.profiler.profile(activities=acts, with_stack=True, with_modules=True)
        with prof:
            yield prof
        os.makedirs(self.output_dir, exist_ok=True)
        prof.export_chrome_trace(os.path.join(self.output_dir, f"trace_rank{self.rank}_{iteration:09d}.json"))

    def trace_path(self, iteration: int) -> Optional[str]:
        return os.path.join(self.output_dir, f"trace_rank{self.rank}_{iteration:09d}.json")
