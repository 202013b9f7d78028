"""Adaptive gradient clipper (reference: ospnext/utils/clip_grads.py:10-124).

Max norm = EMA of the accepted gradient norms + 3σ (EMA of squared deviations);
first step initialises the EMA at ``min(init_max_grad_norm, 3·‖g‖)``; norms above
the threshold are clipped and not folded into the EMA; a non-finite norm raises.

Differences, both deliberate: the global norm is computed once over all local
shards (one all-reduce of a squared sum) instead of ``clip_grad_norm_`` followed
by a second sum over the FSDP group (which counts DTensor norms ``world`` times;
``legacy_group_sum=True`` reproduces that), and the clip factor is returned so
the optimizer can apply it inside the fused AdamW pass instead of rescaling the
gradients in a separate pass.
"""
from __future__ import annotations

import logging
import math
import os
import warnings
from typing import Iterable

import torch
import torch.distributed as dist

GRAD_NORM_INF = 1000.0


def _local(t):
    return t.to_local() if hasattr(t, "to_local") else t


def global_grad_norm(parameters, group=None) -> float:
    grads = [_local(p.grad) for p in parameters if p.grad is not None]
    dev = grads[0].device if grads else torch.device("cpu")
    sq = torch.zeros((), dtype=torch.float32, device=dev)
    if grads:
        norms = torch._foreach_norm([g.float() for g in grads]) if dev.type == "cuda" else [g.float().norm() for g in grads]
        sq = torch.stack([n * n for n in norms]).sum()
    if group is not None and dist.is_initialized():
        # shards are disjoint only inside the FSDP shard group (replicas hold copies)
        sq = sq.reshape(1)
        dist.all_reduce(sq, group=group)
    return float(sq.sqrt().item())


class AdaptiveGradClipper:
    def __init__(self, clip_grad_ema_decay: float = 0.99, init_max_grad_norm: float = 1.0,
                 model_parallel_group=None, legacy_group_sum: bool = False):
        self.clip_grad_ema_decay = clip_grad_ema_decay
        self.model_parallel_group = model_parallel_group
        self.legacy_group_sum = legacy_group_sum
        self.moving_avg_max_grad_norm = -float("inf")
        self.moving_avg_max_grad_norm_var = 0.0
        self.grad_norm_before_clip = 0.0
        self.grad_norm_after_clip = 0.0
        self.max_grad_norm = init_max_grad_norm
        self.max_grad_norm_var = 0.0
        self.save_postfix = "adaptive_grad_clip_states.pt"

    def state_dict(self) -> dict:
        return {k: getattr(self, k) for k in ("clip_grad_ema_decay", "moving_avg_max_grad_norm",
                                              "moving_avg_max_grad_norm_var", "grad_norm_before_clip",
                                              "grad_norm_after_clip", "max_grad_norm", "max_grad_norm_var")}

    def load_state_dict(self, sd: dict):
        for k, v in sd.items():
            setattr(self, k, v)

    def load(self, output_dir: str):
        p = os.path.join(output_dir, self.save_postfix)
        if not os.path.exists(p):
            warnings.warn(f"No adaptive grad clipper state file found at {p}. Use initial values.")
            return
        self.load_state_dict(torch.load(p, map_location="cpu", weights_only=False))

    def save(self, output_dir: str):
        os.makedirs(output_dir, exist_ok=True)
        torch.save(self.state_dict(), os.path.join(output_dir, self.save_postfix))

    @staticmethod
    def get_max_grad_norm(avg, var) -> float:
        return avg + 3.0 * (var ** 0.5)

    @staticmethod
    def get_max_grad_norm_var(avg, g) -> float:
        return (avg - g) ** 2

    def init_weights(self, g0: float):
        self.moving_avg_max_grad_norm = min(self.max_grad_norm, g0 * 3)
        self.moving_avg_max_grad_norm_var = 0.0
        self.max_grad_norm = self.get_max_grad_norm(self.moving_avg_max_grad_norm, 0.0)
        self.max_grad_norm_var = 0.0

    def _norm(self, params) -> float:
        n = global_grad_norm(params, self.model_parallel_group)
        if self.legacy_group_sum and dist.is_initialized():
            n = n * math.sqrt(dist.get_world_size(self.model_parallel_group))
        if not math.isfinite(n):
            raise RuntimeError(f"The total norm for gradients is non-finite ({n}); aborting the step.")
        return n

    def adaptive_clip(self, parameters: Iterable[torch.Tensor], apply: bool = True) -> float:
        """Returns the clip factor; with ``apply`` also scales the gradients in place."""
        params = [parameters] if isinstance(parameters, torch.Tensor) else list(parameters)
        norm = self._norm(params)
        if self.moving_avg_max_grad_norm < -1:
            self.init_weights(norm)
        else:
            self.max_grad_norm = self.get_max_grad_norm(self.moving_avg_max_grad_norm,
                                                        self.moving_avg_max_grad_norm_var)
        self.grad_norm_before_clip = norm
        factor = 1.0
        if norm <= self.max_grad_norm:
            d = self.clip_grad_ema_decay
            self.moving_avg_max_grad_norm = d * self.moving_avg_max_grad_norm + (1 - d) * norm
            self.max_grad_norm_var = self.get_max_grad_norm_var(self.moving_avg_max_grad_norm, norm)
            self.moving_avg_max_grad_norm_var = d * self.moving_avg_max_grad_norm_var + (1 - d) * self.max_grad_norm_var
            self.grad_norm_after_clip = norm
        else:
            factor = self.max_grad_norm / (norm + 1e-6)
            self.grad_norm_after_clip = norm * factor
        if apply and factor != 1.0:
            grads = [_local(p.grad) for p in params if p.grad is not None]
            torch._foreach_mul_(grads, factor)
        return factor
