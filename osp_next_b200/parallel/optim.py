"""AdamW whose update is the fused sm_100a kernel (one launch per parameter shard).

Same update rule and hyper-parameters as ``torch.optim.AdamW`` (the reference's
optimizer, train_osp.py:303-311).  Works on plain tensors and on FSDP2 DTensor
parameters (it updates the local shard).  ``grad_scale`` folds the gradient
clipping factor into the same pass.  CPU tensors fall back to
``torch.optim.AdamW``'s math.
"""
from __future__ import annotations

import torch

from .. import ops


def _local(t):
    return t.to_local() if hasattr(t, "to_local") else t


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.grad_scale = 1.0

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                lp, lg = _local(p.data), _local(p.grad)
                if not st:
                    st["step"] = torch.tensor(0.0)
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
                st["step"] += 1
                step = int(st["step"].item())
                m, v = _local(st["exp_avg"]), _local(st["exp_avg_sq"])
                if lp.is_cuda and lp.dtype == torch.float32 and lp.is_contiguous():
                    ops.adamw_(lp, lg.contiguous(), m, v, group["lr"], b1, b2, group["eps"], group["weight_decay"],
                               step, self.grad_scale)
                else:
                    g = lg.float() * self.grad_scale
                    lp.mul_(1 - group["lr"] * group["weight_decay"])
                    m.mul_(b1).add_(g, alpha=1 - b1)
                    v.mul_(b2).addcmul_(g, g, value=1 - b2)
                    bc1 = 1 - b1 ** step
                    bc2 = 1 - b2 ** step
                    denom = (v.sqrt() / (bc2 ** 0.5)).add_(group["eps"])
                    lp.addcdiv_(m, denom, value=-group["lr"] / bc1)
        return loss
