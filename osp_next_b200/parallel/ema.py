"""Sharded EMA of model parameters (reference: ospnext/distributed/fsdp_ema.py:7-63).

fp32 shadows of the *local* shards (DTensor under FSDP2), updated with
``shadow -= (1−decay)·(shadow − param)`` via foreach kernels; ``store`` /
``restore`` swap live weights for saving / evaluation.  ``lora_only`` restricts
the shadow to LoRA parameters (RL trainer, train_osp_RL.py:905-923).
"""
from __future__ import annotations

import torch
import torch.nn as nn


def _local(t):
    return t.to_local() if hasattr(t, "to_local") else t


class FSDPEMAModel:
    def __init__(self, model: nn.Module, decay: float = 0.9999, update_interval: int = 1, lora_only: bool = False):
        self.decay = decay
        self.one_minus_decay = 1.0 - decay
        self.update_interval = update_interval
        self.lora_only = lora_only
        self.shadow_params = {n: p.detach().clone().float() for n, p in model.named_parameters() if self._keep(n)}
        self.backup = {}

    def _keep(self, name):
        return (not self.lora_only) or ("lora_" in name)

    def get_shadow_params(self):
        return self.shadow_params

    @torch.no_grad()
    def update(self, model: nn.Module, step: int):
        if step % self.update_interval != 0:
            return
        sh, pr, copy_sh, copy_pr = [], [], [], []
        for n, p in model.named_parameters():
            if n not in self.shadow_params:
                continue
            s = _local(self.shadow_params[n])
            lp = _local(p.data)
            if p.requires_grad:
                sh.append(s)
                pr.append(lp.float() if lp.dtype != torch.float32 else lp)
            else:
                copy_sh.append(s)
                copy_pr.append(lp)
        if sh:
            diff = torch._foreach_sub(sh, pr)
            torch._foreach_mul_(diff, self.one_minus_decay)
            torch._foreach_sub_(sh, diff)
        for s, p in zip(copy_sh, copy_pr):
            s.copy_(p)

    @torch.no_grad()
    def ema_copy_to_model(self, model):
        for n, p in model.named_parameters():
            if n in self.shadow_params:
                p.data.copy_(self.shadow_params[n].data)

    @torch.no_grad()
    def model_copy_to_ema(self, model):
        for n, p in model.named_parameters():
            if n in self.shadow_params:
                self.shadow_params[n].data.copy_(p.data)

    def store(self, model):
        self.backup = {n: p.detach().clone() for n, p in model.named_parameters() if n in self.shadow_params}

    @torch.no_grad()
    def restore(self, model):
        for n, p in model.named_parameters():
            if n in self.backup:
                p.data.copy_(self.backup[n].data)
        self.backup = {}
