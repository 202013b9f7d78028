"""LoRA adapters with PEFT-compatible names (reference: train_osp_RL.py:840-903, merge_lora_weights.py).

``inject_lora(model, r, alpha, target_modules)`` replaces each targeted
``nn.Linear`` by :class:`LoraLinear` whose parameters are named like PEFT's
``lora.Linear``: ``<name>.base_layer.{weight,bias}``,
``<name>.lora_A.default.weight`` [r, in], ``<name>.lora_B.default.weight`` [out, r].
Wrapped in :class:`LoraModel`, full parameter names become
``base_model.model.blocks.0.self_attn.q.lora_A.default.weight`` — the key layout
of the reference's ``adapter_model.bin``.  Forward: ``base(x) + B(A(x))·α/r``;
initialisation gaussian A (std 1/r), zero B (PEFT ``init_lora_weights="gaussian"``).
``disable_adapter()`` switches the branch off (reference KL model); ``merge()``
folds ``W += (α/r)·B·A`` (merge_and_unload).
"""
from __future__ import annotations

import contextlib
import fnmatch
import json
import os
from typing import Dict, Iterable, List, Optional

import torch
import torch.nn as nn

from . import functional as Fn


class LoraLinear(nn.Module):
    def __init__(self, base: nn.Linear, r: int, alpha: float, adapter: str = "default"):
        super().__init__()
        self.base_layer = base
        self.r = r
        self.lora_alpha = alpha
        self.scaling = alpha / r
        self.adapter = adapter
        dev, dt = base.weight.device, base.weight.dtype
        self.lora_A = nn.ModuleDict({adapter: nn.Linear(base.in_features, r, bias=False, device=dev, dtype=dt)})
        self.lora_B = nn.ModuleDict({adapter: nn.Linear(r, base.out_features, bias=False, device=dev, dtype=dt)})
        self.disabled = False
        self.reset_lora()

    @property
    def weight(self):
        return self.base_layer.weight

    @property
    def bias(self):
        return self.base_layer.bias

    @property
    def in_features(self):
        return self.base_layer.in_features

    @property
    def out_features(self):
        return self.base_layer.out_features

    def reset_lora(self):
        with torch.no_grad():
            nn.init.normal_(self.lora_A[self.adapter].weight, std=1.0 / self.r)
            nn.init.zeros_(self.lora_B[self.adapter].weight)

    def forward(self, x):
        y = self.base_layer(x) if not isinstance(self.base_layer, nn.Linear) else \
            Fn.linear(x, self.base_layer.weight, self.base_layer.bias)
        if self.disabled:
            return y
        a = Fn.linear(x, self.lora_A[self.adapter].weight)
        b = Fn.linear(a, self.lora_B[self.adapter].weight)
        return y + b.to(y.dtype) * self.scaling

    @torch.no_grad()
    def merged_weight(self):
        A = self.lora_A[self.adapter].weight.float()
        B = self.lora_B[self.adapter].weight.float()
        return (self.base_layer.weight.float() + self.scaling * (B @ A)).to(self.base_layer.weight.dtype)


def _match(name: str, targets: Iterable[str]) -> bool:
    for t in targets:
        if name == t or name.endswith("." + t) or fnmatch.fnmatch(name, t):
            return True
    return False


def inject_lora(model: nn.Module, r: int, alpha: float, target_modules: List[str]) -> List[str]:
    """Replace targeted Linears in place; returns the wrapped module names."""
    done = []
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if isinstance(child, nn.Linear) and _match(full, target_modules):
                setattr(mod, cname, LoraLinear(child, r, alpha))
                done.append(full)
    return done


class LoraModel(nn.Module):
    """PEFT-shaped wrapper: ``self.base_model.model`` is the original network."""

    def __init__(self, model: nn.Module, r: int = 64, lora_alpha: float = 64, target_modules=None,
                 init_lora_weights: str = "gaussian"):
        super().__init__()
        target_modules = list(target_modules or ["q", "k", "v", "o"])
        self.base_model = nn.Module()
        self.base_model.model = model
        self.targets = inject_lora(model, r, lora_alpha, target_modules)
        self.peft_config = {"default": {"r": r, "lora_alpha": lora_alpha, "target_modules": target_modules,
                                        "init_lora_weights": init_lora_weights, "peft_type": "LORA"}}
        for n, p in self.named_parameters():
            p.requires_grad_("lora_" in n)

    def forward(self, *a, **k):
        return self.base_model.model(*a, **k)

    @property
    def model(self):
        return self.base_model.model

    def lora_modules(self):
        return [m for m in self.modules() if isinstance(m, LoraLinear)]

    @contextlib.contextmanager
    def disable_adapter(self):
        mods = self.lora_modules()
        for m in mods:
            m.disabled = True
        try:
            yield
        finally:
            for m in mods:
                m.disabled = False

    def lora_state_dict(self) -> Dict[str, torch.Tensor]:
        """LoRA parameters as full tensors.  Under FSDP2 the parameters are sharded DTensors
        and gathering them is a collective: every rank of the mesh must call this."""
        out = {}
        for n, p in self.named_parameters():
            if "lora_" in n:
                t = p.detach()
                out[n] = t.full_tensor() if hasattr(t, "full_tensor") else t
        return out

    def save_pretrained(self, path: str, write: bool = True):
        """Write ``adapter_model.bin`` + ``adapter_config.json`` (PEFT layout).  Call on every
        rank when the model is FSDP-sharded; only ranks with ``write`` touch the disk."""
        sd = {k: v.cpu().clone() for k, v in self.lora_state_dict().items()}
        if not write:
            return
        os.makedirs(path, exist_ok=True)
        torch.save(sd, os.path.join(path, "adapter_model.bin"))
        with open(os.path.join(path, "adapter_config.json"), "w") as f:
            json.dump(self.peft_config["default"], f, indent=2)

    def load_adapter(self, path: str, strict: bool = True):
        sd = torch.load(os.path.join(path, "adapter_model.bin"), map_location="cpu", weights_only=True)
        own = dict(self.named_parameters())
        missing = [k for k in own if "lora_" in k and k not in sd]
        if strict and missing:
            raise KeyError(f"missing LoRA keys: {missing[:4]}…")
        with torch.no_grad():
            for k, v in sd.items():
                if k in own:
                    own[k].copy_(v.to(own[k].dtype))
        return missing

    @classmethod
    def from_pretrained(cls, model: nn.Module, path: str):
        with open(os.path.join(path, "adapter_config.json")) as f:
            cfg = json.load(f)
        m = cls(model, r=cfg["r"], lora_alpha=cfg["lora_alpha"], target_modules=cfg["target_modules"])
        m.load_adapter(path)
        return m

    @torch.no_grad()
    def merge_and_unload(self) -> nn.Module:
        """Fold every adapter into its base weight and return the plain network."""
        model = self.base_model.model
        for name, mod in list(model.named_modules()):
            for cname, child in list(mod.named_children()):
                if isinstance(child, LoraLinear):
                    base = child.base_layer
                    base.weight.copy_(child.merged_weight())
                    setattr(mod, cname, base)
        return model
