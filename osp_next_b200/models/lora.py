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

    def forward(self, x, act=None):
        if (x.is_cuda and not self.disabled and type(self.base_layer) is nn.Linear
                and not self.base_layer.weight.requires_grad and torch.is_grad_enabled()):
            # trainable adapter on a frozen base (RL / LoRA fine-tuning): one dual GEMM
            return _LoraDualFn.apply(x, self.base_layer.weight, self.base_layer.bias,
                                     self.lora_A[self.adapter].weight, self.lora_B[self.adapter].weight,
                                     self.scaling, act)
        y = self.base_layer(x) if not isinstance(self.base_layer, nn.Linear) else \
            Fn.linear(x, self.base_layer.weight, self.base_layer.bias)
        if not self.disabled:
            a = Fn.linear(x, self.lora_A[self.adapter].weight)
            b = Fn.linear(a, self.lora_B[self.adapter].weight)
            y = y + b.to(y.dtype) * self.scaling
        return Fn.F.gelu(y, approximate="tanh") if act == "gelu_tanh" else y

    @torch.no_grad()
    def merged_weight(self):
        A = self.lora_A[self.adapter].weight.float()
        B = self.lora_B[self.adapter].weight.float()
        return (self.base_layer.weight.float() + self.scaling * (B @ A)).to(self.base_layer.weight.dtype)


class _LoraDualFn(torch.autograd.Function):
    """y = act(x·Wᵀ + b + s·(x·Aᵀ)·Bᵀ) for a frozen base W and trainable A [r, K], B [N, r]:
    forward = the small GEMM a = x·Aᵀ and ONE GEMM with (a, s·B) as a second operand pair
    (GELU in its epilogue when asked); backward with tcgen05 GEMMs:
    g_a = s·gy·B, dA = g_aᵀ·x, dB = s·gyᵀ·a, dX = gy·W + g_a·A."""

    @staticmethod
    def forward(ctx, x, w, bias, A, Bm, scaling, act):
        from .. import ops
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).to(torch.bfloat16)
        a = ops.linear(x2, A.to(torch.bfloat16), None)                     # [M, r] bf16
        sB = (Bm.float() * scaling).to(torch.bfloat16)
        if act == "gelu_tanh":
            y, pre = ops.linear_gelu_aux(x2, w, bias, extra=(a, sB))        # GELU in the epilogue
        else:
            pre = None
            y = ops.linear(x2, w, bias, None, extra=(a, sB))
        ctx.save_for_backward(x2, w, A, Bm, a, pre)
        ctx.meta = (scaling, act, shp, x.dtype, bias is not None)
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        from .. import ops
        x2, w, A, Bm, a, pre = ctx.saved_tensors
        s, act, shp, xdt, has_b = ctx.meta
        g = gy.reshape(-1, gy.shape[-1])
        if act == "gelu_tanh":
            g = ops.gelu_tanh_bwd(g, pre)
        gb = g.to(torch.bfloat16)
        Bb = Bm.to(torch.bfloat16)
        # g_a = s·g·B  [M, r]: B [N, r] read MN-major
        g_a = ops.gemm_t(gb, Bb, a_mn=False, b_mn=True)
        if g_a is None:
            g_a = ops.linear(gb, Bb.t().contiguous(), None, out_dtype=torch.float32)
        g_a = g_a * s
        gab = g_a.to(torch.bfloat16)
        dA = ops.gemm_t(gab, x2, a_mn=True, b_mn=True)
        if dA is None:
            dA = ops.linear(gab.t().contiguous(), x2.t().contiguous(), None, out_dtype=torch.float32)
        dB = ops.gemm_t(gb, a, a_mn=True, b_mn=True)
        if dB is None:
            dB = ops.linear(gb.t().contiguous(), a.t().contiguous(), None, out_dtype=torch.float32)
        dB = dB * s
        dx = None
        if ctx.needs_input_grad[0]:
            dx = ops.gemm_t(gb, w.to(torch.bfloat16), a_mn=False, b_mn=True)
            if dx is None:
                dx = ops.linear(gb, w.to(torch.bfloat16).t().contiguous(), None, out_dtype=torch.float32)
            dxa = ops.gemm_t(gab, A.to(torch.bfloat16), a_mn=False, b_mn=True)
            if dxa is None:
                dxa = ops.linear(gab, A.to(torch.bfloat16).t().contiguous(), None, out_dtype=torch.float32)
            dx = (dx.float() + dxa.float()).view(shp).to(xdt)
        return dx, None, None, dA.to(A.dtype), dB.to(Bm.dtype), None, None


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


# ---------------------------------------------------------------------------- fused inference path
_PACK_CACHE: Dict[tuple, tuple] = {}


def _key(ts):
    return tuple((t.data_ptr(), t._version) for t in ts if t is not None)


def fused_lora_operands(mods, x2d: torch.Tensor):
    """Operands of ONE GEMM computing ``[m_1(x) | … | m_n(x)]`` for Linears / LoraLinears that
    share the input ``x2d`` [M, K]:  base weights concatenated [ΣN, K] + bias, and the LoRA
    branches as a second operand pair ``(a2, b2)`` with ``a2 = x·[A_1; …]ᵀ`` [M, Σr] (one
    small GEMM) and ``b2`` the block-diagonal of ``scaling_i·B_i`` [ΣN, Σr] — so the LoRA
    update accumulates into the base GEMM's accumulator and every fused epilogue still
    applies.  Returns (W, b, extra-or-None); no-grad use (rollouts, inference)."""
    from .. import ops
    base = [m.base_layer if isinstance(m, LoraLinear) else m for m in mods]
    lora = [m for m in mods if isinstance(m, LoraLinear) and not m.disabled]
    wkey = ("w",) + _key([b.weight for b in base] + [b.bias for b in base])
    hit = _PACK_CACHE.get(wkey)
    if hit is None:
        W = torch.cat([b.weight.detach() for b in base], 0).to(torch.bfloat16).contiguous() if len(base) > 1 \
            else base[0].weight.detach().to(torch.bfloat16).contiguous()
        bs = [b.bias for b in base]
        bias = torch.cat([b.detach().float() for b in bs], 0).contiguous() if all(b is not None for b in bs) else None
        hit = (W, bias)
        if len(_PACK_CACHE) > 512:
            _PACK_CACHE.clear()
        _PACK_CACHE[wkey] = hit
    W, bias = hit
    if not lora:
        return W, bias, None
    akey = ("a",) + tuple(id(m) for m in mods) + _key([m.lora_A[m.adapter].weight for m in lora] +
                                                      [m.lora_B[m.adapter].weight for m in lora])
    hit = _PACK_CACHE.get(akey)
    if hit is None:
        A = torch.cat([m.lora_A[m.adapter].weight.detach() for m in lora], 0).to(torch.bfloat16).contiguous()
        rs = sum(m.r for m in lora)
        Bd = torch.zeros(W.shape[0], rs, dtype=torch.bfloat16, device=W.device)
        row = col = 0
        for m in mods:
            n_out = (m.base_layer if isinstance(m, LoraLinear) else m).weight.shape[0]
            if isinstance(m, LoraLinear) and not m.disabled:
                Bd[row:row + n_out, col:col + m.r] = (m.lora_B[m.adapter].weight.detach().float() * m.scaling).to(
                    torch.bfloat16)
                col += m.r
            row += n_out
        hit = (A, Bd)
        _PACK_CACHE[akey] = hit
    A, Bd = hit
    a2 = ops.linear(x2d, A, None)
    return W, bias, (a2, Bd)
