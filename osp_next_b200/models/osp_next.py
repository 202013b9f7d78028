"""OSP-Next DiT: Wan-2.1-shaped transformer with Skiparse-2D sparse blocks.

Parameter names and shapes equal the reference's (ospnext/modules/osp_next.py:
1025-1376, want2v.py:262-287) so Wan-2.1 / OSP-Next checkpoints load unchanged:
``patch_embedding``, ``text_embedding.{0,2}``, ``time_embedding.{0,2}``,
``time_projection.1``, ``blocks.{i}.{norm3, modulation, self_attn.{q,k,v,o,norm_q,
norm_k}, cross_attn.{…}, ffn.{0,2}}``, ``head.{head, modulation}``.

What differs from the reference is *how* a block runs (the math is the same):

* the residual stream of a rank is the ordered token list of its current
  :class:`~osp_next_b200.models.layout.TokenLayout`; Skiparse groups are
  contiguous attention segments, never a permuted copy of the batch, and the
  layout change between Token and Group blocks is stored directly by the
  FFN-down GEMM epilogue (single GPU) or by the SSP exchange (several GPUs);
* q/k/v come from one fused GEMM with a concatenated ``[3C, C]`` weight, followed
  by one fused full-row RMSNorm + 3-D RoPE pass;
* cond/uncond CFG passes run as one batch of 2 (or on two GPU sets);
* the residual stream is fp32 and the time modulation is computed in fp32.
"""
from __future__ import annotations

import functools
import math
from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch
import torch.nn as nn
import torch.utils.checkpoint

from ..utils.profiling import nvtx_range
from . import functional as Fn
from .layout import (FULL, GROUP, TOKEN, ParallelSpec, TokenLayout, block_schedule,
                     make_layout, make_redistribution, token_positions)
from ..ops import reference as ref


# ----------------------------------------------------------------------------- helpers

def sinusoidal_embedding_1d(dim: int, position: torch.Tensor) -> torch.Tensor:
    """``[cos, sin](t·10000^(−i/half))`` computed in float64 (want2v.py:17-28)."""
    assert dim % 2 == 0
    half = dim // 2
    position = position.type(torch.float64)
    idx = torch.arange(half, device=position.device, dtype=torch.float64)
    sinusoid = torch.outer(position, torch.pow(10000, -idx.div(half)))
    return torch.cat([torch.cos(sinusoid), torch.sin(sinusoid)], dim=1)


class WanRMSNorm(nn.Module):
    """RMSNorm over the full row with an fp32 weight (want2v.py:77-93)."""

    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x, weight_only: bool = False):
        if weight_only:
            # the weight as a differentiable tensor produced inside this module's forward:
            # under FSDP the module's own hooks gather the parameter for the call and reduce
            # its gradient afterwards, so a fused kernel elsewhere can consume it
            return self.weight * 1.0
        return Fn.rms_norm(x, self.weight, self.eps)

    def reset_parameters(self):
        nn.init.ones_(self.weight)


class WanLayerNorm(nn.LayerNorm):
    """LayerNorm computed in fp32 (want2v.py:96-106)."""

    def __init__(self, dim, eps=1e-6, elementwise_affine=False):
        super().__init__(dim, elementwise_affine=elementwise_affine, eps=eps)

    def forward(self, x):
        return Fn.layer_norm(x, self.weight, self.bias, self.eps)


@dataclass
class BlockContext:
    """Everything a block needs besides its weights, for one forward pass."""
    layout: TokenLayout
    pos: torch.Tensor                 # int32 [n_local, 3] true (t,h,w) of each local row
    seg: torch.Tensor                 # int32 attention segments over layout.attn_tokens
    freqs: torch.Tensor               # fp32 RoPE angle table
    ulysses_group: object = None      # process group for the head all-to-all (None: none)
    next_dest_row: Optional[torch.Tensor] = None   # fuse the layout change into FFN-down (1 GPU)
    next_n: int = 0
    relaid: bool = False              # set when the block stored its output in the next layout
    p2p: Optional[tuple] = None       # (peer pointer table, dest_rank, dest_row, n_stride): fused SSP exchange
    exchange: object = None           # P2PExchange: Ulysses all-to-all over NVLink instead of NCCL
    ulysses_grp: Optional[tuple] = None   # (size, my index, first rank, splits) of the Ulysses group


class OSPNextSelfAttention(nn.Module):
    def __init__(self, dim, num_heads, window_size=(-1, -1), qk_norm=True, eps=1e-6, **kwargs):
        super().__init__()
        assert dim % num_heads == 0
        self.dim = dim
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.window_size = window_size
        self.qk_norm = qk_norm
        self.eps = eps
        make_linear = kwargs.get("make_linear", nn.Linear)
        self.q = make_linear(dim, dim)
        self.k = make_linear(dim, dim)
        self.v = make_linear(dim, dim)
        self.o = make_linear(dim, dim)
        self.norm_q = WanRMSNorm(dim, eps=eps) if qk_norm else nn.Identity()
        self.norm_k = WanRMSNorm(dim, eps=eps) if qk_norm else nn.Identity()
        self._packed = None
        self.quant_attn = kwargs.get("quant_attn")

    # fused [3C, C] weight for the inference path; rebuilt when any source changes
    def packed_qkv(self):
        ws = (self.q.weight, self.k.weight, self.v.weight)
        bs = (self.q.bias, self.k.bias, self.v.bias)
        key = tuple((t.data_ptr(), t._version) for t in ws + bs)
        if self._packed is None or self._packed[0] != key:
            W = torch.cat([w.detach() for w in ws], 0).to(torch.bfloat16).contiguous()
            b = torch.cat([x.detach() for x in bs], 0).float().contiguous()
            self._packed = (key, W, b)
        return self._packed[1], self._packed[2]

    def _qkv(self, x, ctx: BlockContext):
        B, n, _ = x.shape
        H, D = self.num_heads, self.head_dim
        lora = any(hasattr(m, "lora_A") for m in (self.q, self.k, self.v))
        if Fn._fused(x, self.q.weight) and self.qk_norm and not lora and not _hif8(self):
            W, b = self.packed_qkv()
            qkv = Fn.ops.linear(x, W, b)
            return Fn.ops.qk_norm_rope(qkv, self.norm_q.weight, self.norm_k.weight, ctx.pos, ctx.freqs, H, self.eps)
        if (lora and not _hif8(self) and self.qk_norm and ctx.pos is not None
                and Fn._fused(x, self.q.weight, *[p for m in (self.q, self.k, self.v) for p in _lora_params(m)])):
            # LoRA folded into the packed QKV GEMM (second operand pair), then the fused q/k
            # norm + RoPE, as the plain path
            from .lora import fused_lora_operands
            x2 = x.reshape(-1, x.shape[-1])
            W, b, extra = fused_lora_operands((self.q, self.k, self.v), x2)
            qkv = Fn.ops.linear(x2, W, b, extra=extra).view(B, n, -1)
            return Fn.ops.qk_norm_rope(qkv, self.norm_q.weight, self.norm_k.weight, ctx.pos, ctx.freqs, H, self.eps)
        if (x.is_cuda and self.qk_norm and not lora and not _hif8(self) and ctx.pos is not None
                and all(type(m) is nn.Linear for m in (self.q, self.k, self.v))):
            # training: one QKV GEMM + fused q/k norm and RoPE with kernel backward
            return Fn.qkv_norm_rope(x, (self.q.weight, self.k.weight, self.v.weight),
                                    (self.q.bias, self.k.bias, self.v.bias), self.norm_q(None, weight_only=True),
                                    self.norm_k(None, weight_only=True), ctx.pos, ctx.freqs, H, self.eps)
        if x.is_cuda and self.qk_norm and ctx.pos is not None and (D * H) % 4 == 0:
            # wrapped projections (LoRA, HiF8) run their own forward (HiF8: one quantisation of
            # x and one GEMM for all three); the q/k RMSNorm and the RoPE stay on the fused
            # kernel (forward and backward) whatever the Linear type
            if _hif8(self) and all(getattr(m, "is_hif8", False) for m in (self.q, self.k, self.v)):
                from ..quant.hif8 import hif8_multi_linear
                qkv = hif8_multi_linear(x, (self.q, self.k, self.v))
            else:
                qkv = torch.cat([_lin(self.q, x), _lin(self.k, x), _lin(self.v, x)], dim=-1)
            wq = self.norm_q(None, weight_only=True) if torch.is_grad_enabled() else self.norm_q.weight
            wk = self.norm_k(None, weight_only=True) if torch.is_grad_enabled() else self.norm_k.weight
            return Fn.qk_norm_rope_packed(qkv, wq, wk, ctx.pos, ctx.freqs, H, self.eps)
        q = self.norm_q(_lin(self.q, x)).view(B, n, H, D)
        k = self.norm_k(_lin(self.k, x)).view(B, n, H, D)
        v = _lin(self.v, x).view(B, n, H, D)
        q = Fn.apply_rope(q, ctx.pos, ctx.freqs)
        k = Fn.apply_rope(k, ctx.pos, ctx.freqs)
        dt = torch.bfloat16 if x.is_cuda else v.dtype
        return q.to(dt), k.to(dt), v.to(dt)

    def forward(self, x, ctx: BlockContext):
        """x: modulated-normalised input [B, n_local, C] → attention output [B, n_local, C]."""
        q, k, v = self._qkv(x, ctx)
        p2p_ul = ctx.ulysses_group is not None and ctx.exchange is not None and q.is_cuda
        if p2p_ul:                    # one staged NVLink exchange for q, k and v
            from ..parallel.p2p_collectives import p2p_ulysses_scatter
            q, k, v = p2p_ulysses_scatter(ctx.exchange, ctx.ulysses_grp, q, k, v)
        elif ctx.ulysses_group is not None:
            from ..parallel.comm import ulysses_all_to_all
            q = ulysses_all_to_all(q, ctx.ulysses_group, ctx.layout.a2a_splits, True)
            k = ulysses_all_to_all(k, ctx.ulysses_group, ctx.layout.a2a_splits, True)
            v = ulysses_all_to_all(v, ctx.ulysses_group, ctx.layout.a2a_splits, True)
        if self.quant_attn == "hif8":
            from ..quant.hif8 import hif8_qkv
            q, k, v = hif8_qkv(q, k, v, getattr(self, "scale_max_forward", 15.0),
                               getattr(self, "scale_max_backward", 224.0))
        o = Fn.attention(q, k, v, ctx.seg, ctx.seg)
        if p2p_ul:
            from ..parallel.p2p_collectives import p2p_ulysses_gather
            (o,) = p2p_ulysses_gather(ctx.exchange, ctx.ulysses_grp, o)
        elif ctx.ulysses_group is not None:
            from ..parallel.comm import ulysses_all_to_all
            o = ulysses_all_to_all(o, ctx.ulysses_group, ctx.layout.a2a_splits, False)
        return o.flatten(2)


def _hif8(attn) -> bool:
    return getattr(attn.q, "is_hif8", False)


def _lin(mod, x, act=None):
    """Plain Linears go through the functional layer (fused GEMM / dtype handling); LoRA
    Linears without autograd fold their branch into the same GEMM; other wrapped ones
    (HiF8, LoRA under autograd) run their own forward."""
    if type(mod) is nn.Linear:
        return Fn.linear(x, mod.weight, mod.bias, act=act)
    if _lora_fusable(mod, x):
        from .lora import fused_lora_operands
        x2 = x.reshape(-1, x.shape[-1])
        W, b, extra = fused_lora_operands((mod,), x2)
        return Fn.ops.linear(x2, W, b, act=act, extra=extra).view(*x.shape[:-1], W.shape[0])
    y = mod(x)
    return Fn.F.gelu(y, approximate="tanh") if act == "gelu_tanh" else y


def _lora_params(mod):
    return [mod.lora_A[mod.adapter].weight, mod.lora_B[mod.adapter].weight] if hasattr(mod, "lora_A") else []


def _lora_fusable(mod, x) -> bool:
    """A LoRA Linear may take the folded no-grad GEMM only when no autograd graph is needed
    through its input, its base weight or its LoRA factors."""
    return (hasattr(mod, "lora_A") and type(mod.base_layer) is nn.Linear
            and Fn._fused(x, mod.weight, *_lora_params(mod)))


def _gated_out(mod, h, resid, gate, dest_row=None, n_out=None):
    """resid + mod(h)·gate: plain and (no-grad) LoRA Linears on the gated-residual GEMM
    epilogue (optionally storing rows in the next layout), others on the fused gated add."""
    if _plain(mod):
        if dest_row is not None:
            return Fn.ops.linear_gated_residual(h, mod.weight, mod.bias, resid, gate, dest_row=dest_row, n_out=n_out)
        return Fn.gated_residual_linear(h, mod.weight, mod.bias, resid, gate)
    if _lora_fusable(mod, h) and resid.dtype == torch.float32 and Fn._fused(resid):
        from .lora import fused_lora_operands
        W, b, extra = fused_lora_operands((mod,), h.reshape(-1, h.shape[-1]))
        out = resid if (dest_row is None and resid.is_contiguous()) else None
        return Fn.ops.linear_gated_residual(h, W, b, resid, gate, dest_row=dest_row, n_out=n_out, out=out,
                                            extra=extra)
    return Fn.gated_add(resid, mod(h), gate)


class OSPNextCrossAttention(OSPNextSelfAttention):
    def text_kv(self, text):
        B, L, _ = text.shape
        H, D = self.num_heads, self.head_dim
        k = self.norm_k(_lin(self.k, text)).view(B, L, H, D)
        v = _lin(self.v, text).view(B, L, H, D)
        return k, v

    def forward(self, x, text, kv=None):
        B, n, _ = x.shape
        H, D = self.num_heads, self.head_dim
        q = self.norm_q(_lin(self.q, x)).view(B, n, H, D)
        k, v = kv if kv is not None else self.text_kv(text)
        if self.quant_attn == "hif8":
            from ..quant.hif8 import hif8_qkv
            q, k, v = hif8_qkv(q, k, v, getattr(self, "scale_max_forward", 15.0),
                               getattr(self, "scale_max_backward", 224.0))
        seg_q, seg_k = _one_segment(n), _one_segment(k.shape[1])
        if x.is_cuda:
            q, k, v = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)
        return Fn.attention(q, k, v, seg_q, seg_k).flatten(2)


class OSPNextAttentionBlock(nn.Module):
    def __init__(self, dim, ffn_dim, num_heads, window_size=(-1, -1), qk_norm=True, cross_attn_norm=False,
                 eps=1e-6, sparse_ratio=2, skiparse_block_type=FULL, is_full2skiparse_block=False,
                 is_skiparse2full_block=False, quant=None, quant_attn=None, scale_max_forward=15.0,
                 scale_max_backward=224.0):
        super().__init__()
        self.dim = dim
        self.ffn_dim = ffn_dim
        self.num_heads = num_heads
        self.eps = eps
        self.cross_attn_norm = cross_attn_norm
        make_linear = _linear_factory(quant, scale_max_forward, scale_max_backward)
        kw = dict(make_linear=make_linear, quant_attn=quant_attn)
        self.norm1 = WanLayerNorm(dim, eps)
        self.self_attn = OSPNextSelfAttention(dim, num_heads, window_size, qk_norm, eps, **kw)
        self.norm3 = WanLayerNorm(dim, eps, elementwise_affine=True) if cross_attn_norm else nn.Identity()
        self.cross_attn = OSPNextCrossAttention(dim, num_heads, window_size, qk_norm, eps, **kw)
        self.norm2 = WanLayerNorm(dim, eps)
        self.ffn = nn.Sequential(make_linear(dim, ffn_dim), nn.GELU(approximate="tanh"), make_linear(ffn_dim, dim))
        self.modulation = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)
        for a in (self.self_attn, self.cross_attn):
            a.scale_max_forward = scale_max_forward
            a.scale_max_backward = scale_max_backward
        self.sparse_ratio = sparse_ratio
        self.skiparse_block_type = skiparse_block_type
        self.is_full2skiparse_block = is_full2skiparse_block
        self.is_skiparse2full_block = is_skiparse2full_block

    def reset_parameters(self):
        with torch.no_grad():
            self.modulation.copy_(torch.randn_like(self.modulation) / self.dim ** 0.5)

    def block_forward(self, x, e0, text, ctx: BlockContext, text_kv=None):
        e = (self.modulation.float() + e0.float())                      # [B,6,C]
        e = [e[:, i] for i in range(6)]
        # self-attention
        xm = Fn.ln_modulate(x, e[0], e[1], self.eps)
        y = self.self_attn(xm, ctx)
        x = _gated_out(self.self_attn.o, y, x, e[2])
        # cross-attention
        xn = self.norm3(x) if self.cross_attn_norm else (x if not x.is_cuda else x.to(torch.bfloat16))
        y = self.cross_attn(xn, text, text_kv)
        x = _gated_out(self.cross_attn.o, y, x, None)
        # FFN
        xm = Fn.ln_modulate(x, e[3], e[4], self.eps)
        f0, f2 = self.ffn[0], self.ffn[2]
        if getattr(f0, "is_hif8", False):
            from ..quant.hif8 import hif8_multi_linear
            h = hif8_multi_linear(xm, (f0,), act="gelu_tanh")       # GELU in the GEMM epilogue
        elif _plain(f0) or _lora_fusable(f0, xm):
            h = _lin(f0, xm, act="gelu_tanh")
        elif hasattr(f0, "lora_A"):
            h = f0(xm, act="gelu_tanh")                 # LoRA under autograd: GELU in the dual GEMM
        else:
            h = self.ffn[1](f0(xm))
        if _plain(f2) and ctx.p2p is not None and Fn._fused(h, f2.weight, x):
            # fused SSP exchange: every output row goes straight to its owner rank over NVLink
            ptrs, drank, drow, stride = ctx.p2p
            Fn.ops.linear_gated_residual_p2p(h, f2.weight, f2.bias, x, e[5], drank, drow, ptrs, stride)
            ctx.relaid = True
            return None
        if (_plain(f2) or _lora_fusable(f2, h)) and ctx.next_dest_row is not None and Fn._fused(h, f2.weight, x):
            # layout change for the next block fused into the FFN-down store
            ctx.relaid = True
            return _gated_out(f2, h, x, e[5], dest_row=ctx.next_dest_row, n_out=ctx.next_n)
        return _gated_out(f2, h, x, e[5])

    def forward(self, x, e0, text, ctx: BlockContext, text_kv=None, gradient_checkpointing=False):
        if gradient_checkpointing and torch.is_grad_enabled():
            lora = [p for n_, p in self.named_parameters() if "lora_" in n_]

            def run(x_, e0_, text_, *lora_dummy):
                return self.block_forward(x_, e0_, text_, ctx, text_kv)
            return torch.utils.checkpoint.checkpoint(run, x, e0, text, *lora, use_reentrant=False)
        return self.block_forward(x, e0, text, ctx, text_kv)


def _plain(m) -> bool:
    """A plain nn.Linear (no LoRA / HiF8 wrapper) can use the fused GEMM epilogues."""
    return type(m) is nn.Linear


def _linear_factory(quant, smf, smb):
    if quant == "hif8":
        from ..quant.hif8 import HIF8Linear

        def mk(i, o, bias=True):
            return HIF8Linear(i, o, bias=bias, scale_max_forward=smf, scale_max_backward=smb)
        return mk
    return nn.Linear


class Head(nn.Module):
    """Output head: LN + modulation + Linear(C → prod(patch)·out) (want2v.py:262-287)."""

    def __init__(self, dim, out_dim, patch_size, eps=1e-6):
        super().__init__()
        self.dim = dim
        self.out_dim = out_dim
        self.patch_size = patch_size
        self.eps = eps
        self.norm = WanLayerNorm(dim, eps)
        self.head = nn.Linear(dim, math.prod(patch_size) * out_dim)
        self.modulation = nn.Parameter(torch.randn(1, 2, dim) / dim ** 0.5)

    def forward(self, x, e):
        m = self.modulation.float() + e.float()[:, None, :]
        xm = Fn.ln_modulate(x, m[:, 0], m[:, 1], self.eps)
        return Fn.linear(xm, self.head.weight, self.head.bias)


class OSPNextModel(nn.Module):
    """OSP-Next DiT (registry name ``osp_next``)."""

    def __init__(self, model_type="t2v", patch_size=(1, 2, 2), text_len=512, in_dim=16, dim=2048, ffn_dim=8192,
                 freq_dim=256, text_dim=4096, out_dim=16, num_heads=16, num_layers=32, window_size=(-1, -1),
                 qk_norm=True, cross_attn_norm=True, eps=1e-6, skiparse_model_type="full", sparse_ratio=2,
                 num_full_blocks=0, quant=None, quant_attn=None, scale_max_forward=15.0, scale_max_backward=224.0,
                 **kwargs):
        super().__init__()
        assert model_type in ("t2v", "i2v")
        self.model_type = model_type
        self.patch_size = tuple(patch_size)
        self.text_len = text_len
        self.in_dim = in_dim
        self.dim = dim
        self.ffn_dim = ffn_dim
        self.freq_dim = freq_dim
        self.text_dim = text_dim
        self.out_dim = out_dim
        self.num_heads = num_heads
        self.num_layers = num_layers
        self.window_size = window_size
        self.qk_norm = qk_norm
        self.cross_attn_norm = cross_attn_norm
        self.eps = eps
        self.quant = quant
        self.quant_attn = quant_attn
        self.gradient_checkpointing = False
        self.config = dict(model_type=model_type, patch_size=list(self.patch_size), text_len=text_len, in_dim=in_dim,
                           dim=dim, ffn_dim=ffn_dim, freq_dim=freq_dim, text_dim=text_dim, out_dim=out_dim,
                           num_heads=num_heads, num_layers=num_layers, qk_norm=qk_norm,
                           cross_attn_norm=cross_attn_norm, eps=eps, skiparse_model_type=skiparse_model_type,
                           sparse_ratio=sparse_ratio, num_full_blocks=num_full_blocks, quant=quant,
                           quant_attn=quant_attn, scale_max_forward=scale_max_forward,
                           scale_max_backward=scale_max_backward)

        self.patch_embedding = nn.Conv3d(in_dim, dim, kernel_size=patch_size, stride=patch_size)
        self.text_embedding = nn.Sequential(nn.Linear(text_dim, dim), nn.GELU(approximate="tanh"), nn.Linear(dim, dim))
        self.time_embedding = nn.Sequential(nn.Linear(freq_dim, dim), nn.SiLU(), nn.Linear(dim, dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(dim, dim * 6))

        self.skiparse_model_type = skiparse_model_type
        self.sparse_ratio = 1 if skiparse_model_type == "full" else sparse_ratio
        kinds, full_idx = block_schedule(num_layers, skiparse_model_type, num_full_blocks)
        self.num_full_blocks = len(full_idx)
        self.block_kinds = kinds
        self.full_block_indices = full_idx
        self.blocks = nn.ModuleList()
        for i, kind in enumerate(kinds):
            prev_full = i == 0 or kinds[i - 1] == FULL
            next_full = i == num_layers - 1 or kinds[i + 1] == FULL
            self.blocks.append(OSPNextAttentionBlock(
                dim, ffn_dim, num_heads, window_size, qk_norm, cross_attn_norm, eps,
                sparse_ratio=self.sparse_ratio if kind != FULL else 1, skiparse_block_type=kind,
                is_full2skiparse_block=kind != FULL and prev_full, is_skiparse2full_block=kind != FULL and next_full,
                quant=quant, quant_attn=quant_attn, scale_max_forward=scale_max_forward,
                scale_max_backward=scale_max_backward))
        self.head = Head(dim, out_dim, self.patch_size, eps)
        assert dim % num_heads == 0 and (dim // num_heads) % 2 == 0
        self.rope_d = dim // num_heads
        self._freqs = None
        self.parallel: Optional["SPRuntime"] = None      # set by parallel.sp.attach_sp
        self._text_kv_cache = None
        self.init_weights()

    # ------------------------------------------------------------------ misc API
    def set_gradient_checkpointing(self, enabled=False):
        self.gradient_checkpointing = enabled

    def reset_parameters(self):
        self.init_weights()

    def init_weights(self):
        for n, m in self.named_modules():
            if n and hasattr(m, "reset_parameters"):
                m.reset_parameters()

    @property
    def dtype(self):
        return self.patch_embedding.weight.dtype

    def freqs(self, device):
        if self._freqs is None or self._freqs.device != torch.device(device):
            self._freqs = ref.rope_freqs(self.rope_d).to(device)
        return self._freqs

    def enable_text_kv_cache(self, enabled: bool = True):
        """Cache cross-attention K/V of the text per block (constant across sampler steps).

        Entries are keyed by the text tensor's storage; the sampler clears the cache at
        the start of every ``sample`` call so a reused allocation never serves stale K/V.
        """
        self._text_kv_cache = {} if enabled else None

    def reset_text_kv_cache(self):
        if self._text_kv_cache is not None:
            self._text_kv_cache.clear()

    # ------------------------------------------------------------------ embeddings
    def patchify_embed(self, x):
        """Conv3d(k=s=patch) as one GEMM over flattened patches → [B, N, C], grid."""
        B, Cin, T, H, W = x.shape
        pt, ph, pw = self.patch_size
        grid = (T // pt, H // ph, W // pw)
        w = self.patch_embedding.weight
        if not x.is_cuda:
            y = self.patch_embedding(x.to(w.dtype))
            return y.flatten(2).transpose(1, 2), grid
        p = x.view(B, Cin, grid[0], pt, grid[1], ph, grid[2], pw).permute(0, 2, 4, 6, 1, 3, 5, 7)
        p = p.reshape(B, grid[0] * grid[1] * grid[2], Cin * pt * ph * pw).to(torch.bfloat16)
        y = Fn.linear(p, w.reshape(w.shape[0], -1), self.patch_embedding.bias)
        return y.float(), grid

    def unpatchify(self, x, grid):
        """b (f h w) (x y z c) -> b c (f x) (h y) (w z) (osp_next.py:1349-1368)."""
        B = x.shape[0]
        f, h, w = grid
        pt, ph, pw = self.patch_size
        c = self.out_dim
        x = x.view(B, f, h, w, pt, ph, pw, c).permute(0, 7, 1, 4, 2, 5, 3, 6)
        return x.reshape(B, c, f * pt, h * ph, w * pw)

    def time_embed(self, t):
        tf = sinusoidal_embedding_1d(self.freq_dim, t).float()
        te0, te2 = self.time_embedding[0], self.time_embedding[2]
        e = torch.nn.functional.linear(tf, te0.weight.float(), te0.bias.float())
        e = torch.nn.functional.linear(torch.nn.functional.silu(e), te2.weight.float(), te2.bias.float())
        tp = self.time_projection[1]
        e0 = torch.nn.functional.linear(torch.nn.functional.silu(e), tp.weight.float(), tp.bias.float())
        return e, e0.unflatten(1, (6, self.dim))

    def text_embed(self, text):
        l0, l2 = self.text_embedding[0], self.text_embedding[2]
        h = Fn.linear(text.to(l0.weight.dtype) if not text.is_cuda else text, l0.weight, l0.bias, act="gelu_tanh")
        return Fn.linear(h, l2.weight, l2.bias)

    # ------------------------------------------------------------------ forward
    def forward(self, x, t, text, **kwargs):
        """x [B,C,T,H,W] latents, t [B] timesteps (σ·1000), text [B,L,text_dim] → velocity fp32."""
        device = x.device
        x, grid = self.patchify_embed(x)
        e, e0 = self.time_embed(t.to(device))
        text = self.text_embed(text)
        rt = self.parallel
        spec = rt.spec if rt is not None else ParallelSpec()
        P = self.sparse_ratio
        freqs = self.freqs(device)

        prev_kind = None
        # rows of the first layout (every rank computed the full patch embedding)
        first = make_layout(self.block_kinds[0], grid, P, spec)
        x = x[:, _dev(first.tokens, device, torch.long)] if not _is_arange(first.tokens, x.shape[1]) else x
        prev_kind = self.block_kinds[0]
        nb = len(self.blocks)
        for i, block in enumerate(self.blocks):
            kind = self.block_kinds[i]
            if kind != prev_kind:
                x = self._redistribute(x, prev_kind, kind, grid, spec)
            prev_kind = kind
            ctx = self._context(kind, grid, spec, device, freqs)
            nxt = self.block_kinds[i + 1] if i + 1 < nb else None
            fuse = (spec.world == 1 and nxt is not None and nxt != kind and x.is_cuda
                    and not (torch.is_grad_enabled() and self.training))
            if fuse:
                rd = make_redistribution(kind, nxt, grid, P, spec)
                ctx.next_dest_row = _dev(rd.dest_row, device, torch.int32)
                ctx.next_n = rd.n_out
            p2p = getattr(rt, "p2p", None) if rt is not None else None
            use_p2p = (p2p is not None and spec.world > 1 and spec.full_sp == spec.world and nxt is not None
                       and nxt != kind and x.is_cuda and not torch.is_grad_enabled())
            if use_p2p:
                rd = make_redistribution(kind, nxt, grid, P, spec)
                ctx.p2p = (p2p.target(), _dev(rd.dest_rank, device, torch.int32),
                           _dev(rd.dest_row, device, torch.int32), p2p.n_stride)
            kv = None
            if self._text_kv_cache is not None and not torch.is_grad_enabled():
                key = (i, text.data_ptr(), text.shape)
                kv = self._text_kv_cache.get(key)
                if kv is None:
                    kv = block.cross_attn.text_kv(text)
                    self._text_kv_cache[key] = kv
            with nvtx_range(f"block{i}_{kind}"):
                x = block(x, e0, text, ctx, kv, gradient_checkpointing=self.gradient_checkpointing)
            if ctx.relaid:                   # the FFN-down epilogue already stored the next layout
                if ctx.p2p is not None:      # peers wrote into our buffer: order, then read it
                    p2p.barrier()
                    x = p2p.take(rd.n_out)
                prev_kind = nxt
        x = self.head(x, e)
        # back to natural order, full sequence on every rank
        x = self._gather_natural(x, prev_kind, grid, spec)
        return self.unpatchify(x, grid).float()

    def _context(self, kind, grid, spec, device, freqs) -> BlockContext:
        lay = make_layout(kind, grid, self.sparse_ratio, spec)
        pos = _dev(_layout_positions(kind, tuple(grid), self.sparse_ratio, spec), device, torch.int32)
        seg = lay.seg
        ug, ex, grp = None, None, None
        if lay.a2a_splits is not None and self.parallel is not None:
            dense = kind == FULL or self.sparse_ratio == 1
            ug = self.parallel.full_group if dense else self.parallel.ulysses_group
            ex = getattr(self.parallel, "p2p", None)
            if ex is not None:
                from ..parallel.p2p_collectives import ulysses_group_of
                grp = ulysses_group_of(spec, dense) + (tuple(lay.a2a_splits),)
        return BlockContext(layout=lay, pos=pos, seg=seg, freqs=freqs, ulysses_group=ug, exchange=ex,
                            ulysses_grp=grp)

    def _redistribute(self, x, ka, kb, grid, spec):
        rd = make_redistribution(ka, kb, grid, self.sparse_ratio, spec)
        if spec.world == 1:
            return x if rd.identity else x[:, _dev(rd.gather, x.device, torch.long)]
        ex = getattr(self.parallel, "p2p", None)
        if ex is not None and x.is_cuda:
            from ..parallel.p2p_collectives import p2p_redistribute
            return p2p_redistribute(x, ka, kb, grid, self.sparse_ratio, spec, ex)
        from ..parallel.redistribute import redistribute
        return redistribute(x, rd, self.parallel.global_sp_group)

    def _gather_natural(self, x, kind, grid, spec):
        lay = make_layout(kind, grid, self.sparse_ratio, spec)
        N = grid[0] * grid[1] * grid[2]
        if spec.world == 1:
            if _is_arange(lay.tokens, N):
                return x
            out = x.new_empty(x.shape[0], N, x.shape[2])
            out[:, _dev(lay.tokens, x.device, torch.long)] = x
            return out
        from ..parallel.redistribute import gather_natural
        return gather_natural(x, kind, grid, self.sparse_ratio, spec, self.parallel.global_sp_group)


def _is_arange(idx: torch.Tensor, n: int) -> bool:
    return idx.numel() == n and bool(torch.equal(idx, torch.arange(n, dtype=idx.dtype)))


_DEV_CACHE = {}


@functools.lru_cache(maxsize=256)
def _layout_positions(kind, grid, P, spec) -> torch.Tensor:
    """(t, h, w) of a layout's tokens; one CPU tensor per layout, so its device copy is cached."""
    return token_positions(make_layout(kind, grid, P, spec).tokens, grid)


@functools.lru_cache(maxsize=64)
def _one_segment(n: int) -> torch.Tensor:
    """Segment table [0, n] (one CPU tensor per length, so its device copy is cached)."""
    return torch.tensor([0, n], dtype=torch.int32)


def _dev(t: torch.Tensor, device, dtype):
    key = (id(t), str(device), dtype)
    v = _DEV_CACHE.get(key)
    if v is None or v[0] is not t:
        if len(_DEV_CACHE) > 4096:       # inputs are cached host tables; bound it all the same
            _DEV_CACHE.clear()
        v = (t, t.to(device=device, dtype=dtype))
        _DEV_CACHE[key] = v
    return v[1]


models = {"osp_next": OSPNextModel}
models_main_block = {"osp_next": OSPNextAttentionBlock}
models_blocks_to_float = {"osp_next": [WanLayerNorm, WanRMSNorm]}
models_blocks_to_output_float = {"osp_next": None}


def _save_pretrained(self, path, **kw):
    from .pretrained import save_pretrained
    return save_pretrained(self, path, **kw)


@classmethod
def _from_pretrained(cls, path, **kw):
    from .pretrained import from_pretrained
    return from_pretrained(cls, path, **kw)


OSPNextModel.save_pretrained = _save_pretrained
OSPNextModel.from_pretrained = _from_pretrained
