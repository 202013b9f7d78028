"""Functional layer the DiT modules call.

Three paths, chosen per call:

* CPU tensors: plain differentiable PyTorch in the tensors' own dtype — the
  reference's math without autocast, so fp32 CPU runs compare bit-for-bit-ish
  with the reference model (tests/test_parity_reference.py).
* CUDA, no autograd (sampling, RL rollouts): the fused sm_100a kernels of
  :mod:`osp_next_b200.ops` (bf16 operands, fp32 accumulation, fp32 residual).
* CUDA with autograd (training): :class:`torch.autograd.Function` wrappers whose
  forward runs the same kernels; GEMM backward runs on the same tcgen05 GEMM
  (reading dY, W and X MN-major in place); attention backward on its own tcgen05
  kernels; LN-modulate, RMSNorm, q/k-norm + RoPE, gated residual and GELU backward on
  fused kernels (``ops/csrc/train_ops.cu``).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref

_BF16 = torch.bfloat16


def _fused(*ts) -> bool:
    """Fused kernel path: CUDA tensors and no autograd graph being built."""
    t0 = next(t for t in ts if t is not None)
    if not t0.is_cuda:
        return False
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts):
        return False
    return True


def _grad_cuda(*ts) -> bool:
    t0 = next(t for t in ts if t is not None)
    return t0.is_cuda and not _fused(*ts)


# ----------------------------------------------------------------------------- GEMM autograd

class _LinearFn(torch.autograd.Function):
    """y = act(x·Wᵀ + b) with forward and backward GEMMs on the tcgen05 kernel."""

    @staticmethod
    def forward(ctx, x, w, b, act):
        x2 = x.reshape(-1, x.shape[-1]).to(_BF16)
        wb = w.to(_BF16)
        if act == "gelu_tanh" and w.shape[0] % 32 == 0 and x2.shape[1] % 8 == 0:
            # one GEMM writes gelu(pre) and pre (bf16, as the reference's autocast Linear output)
            y, pre = ops.linear_gelu_aux(x2, wb, b)
            ctx.save_for_backward(x2, wb, pre)
        elif act == "gelu_tanh":
            pre = ops.linear(x2, wb, b, None, out_dtype=torch.float32)
            y = F.gelu(pre, approximate="tanh").to(_BF16)
            ctx.save_for_backward(x2, wb, pre)
        else:
            y = ops.linear(x2, wb, b, None)
            ctx.save_for_backward(x2, wb, None)
        ctx.act = act
        ctx.has_b = b is not None
        ctx.in_shape = x.shape
        ctx.w_dtype = w.dtype
        ctx.x_dtype = x.dtype
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, wb, pre = ctx.saved_tensors
        g = gy.reshape(-1, gy.shape[-1])
        if ctx.act == "gelu_tanh" and pre.dtype == _BF16:
            g = ops.gelu_tanh_bwd(g, pre)
        elif ctx.act == "gelu_tanh":
            with torch.enable_grad():
                p = pre.detach().requires_grad_(True)
                out = F.gelu(p, approximate="tanh")
                (g,) = torch.autograd.grad(out, p, g.float())
        gb = g.to(_BF16)
        # dX = dY·W: W read MN-major in place; dW = dYᵀ·X: dY and X read MN-major in place
        dx_dtype = _BF16 if ctx.x_dtype == _BF16 else torch.float32
        dx = ops.gemm_t(gb, wb, a_mn=False, b_mn=True, out_dtype=dx_dtype)
        if dx is None:
            dx = ops.linear(gb, wb.t().contiguous(), None, None, out_dtype=torch.float32)
        # a bf16 weight takes its gradient in bf16 straight from the GEMM epilogue (the same
        # fp32 accumulation rounded once), skipping an fp32 write and a conversion pass
        dw_dtype = _BF16 if ctx.w_dtype == _BF16 else torch.float32
        dw = ops.gemm_t(gb, x2, a_mn=True, b_mn=True, out_dtype=dw_dtype)
        if dw is None:
            dw = ops.linear(gb.t().contiguous(), x2.t().contiguous(), None, None, out_dtype=torch.float32)
        db = ops.bias_grad(g) if ctx.has_b else None
        return dx.view(ctx.in_shape).to(ctx.x_dtype), dw.to(ctx.w_dtype), db, None


class _GatedAddFn(torch.autograd.Function):
    """out = resid + y·gate[b] (fp32 residual, bf16 branch output), fused fwd/bwd kernels."""

    @staticmethod
    def forward(ctx, resid, y, gate):
        ctx.save_for_backward(y, gate)
        ctx.has_gate = gate is not None
        return ops.gated_add(resid, y, gate)

    @staticmethod
    def backward(ctx, dout):
        y, gate = ctx.saved_tensors
        dout = dout.float().contiguous()
        if not ctx.has_gate:
            return dout, dout.to(_BF16), None
        dy, dgate = ops.gated_add_bwd(dout, y, gate)
        return dout, dy, dgate.to(gate.dtype)


class _LNModFn(torch.autograd.Function):
    """bf16 LN(x)·(1+scale[b]) + shift[b] of the fp32 residual, fused fwd/bwd kernels."""

    @staticmethod
    def forward(ctx, x, shift, scale, eps):
        ctx.save_for_backward(x, scale)
        ctx.eps = eps
        return ops.ln_modulate(x, shift, scale, eps)

    @staticmethod
    def backward(ctx, dy):
        x, scale = ctx.saved_tensors
        dx, dsc, dsh = ops.ln_modulate_bwd(x, dy, scale, ctx.eps)
        return dx, dsh, dsc, None


class _QKNormRopeFn(torch.autograd.Function):
    """Full-row RMSNorm of q and k + 3-D RoPE on a fused qkv [B,n,3C] (out of place)."""

    @staticmethod
    def forward(ctx, qkv, wq, wk, pos, freqs, num_heads, eps):
        C = qkv.shape[-1] // 3
        raw = qkv[..., :2 * C].contiguous()
        out = qkv.contiguous().clone()
        ops.qk_norm_rope(out, wq, wk, pos, freqs, num_heads, eps)
        ctx.save_for_backward(raw, wq, wk, pos, freqs)
        ctx.eps = eps
        ctx.D = C // num_heads
        return out

    @staticmethod
    def backward(ctx, gout):
        raw, wq, wk, pos, freqs = ctx.saved_tensors
        C = raw.shape[-1] // 2
        B, n = raw.shape[:2]
        H = C // ctx.D
        sh = (B, n, H, ctx.D)
        dq, dk, dv = gout[..., :C].reshape(sh), gout[..., C:2 * C].reshape(sh), gout[..., 2 * C:].reshape(sh)
        dqkv, dwq, dwk = ops.qk_norm_rope_bwd(raw, dq, dk, dv, wq, wk, pos, freqs, ctx.eps)
        return dqkv, dwq.to(wq.dtype), dwk.to(wk.dtype), None, None, None, None


def qkv_norm_rope(x, ws, bs, wq_norm, wk_norm, pos, freqs, num_heads: int, eps: float):
    """Training path of the self-attention input: one GEMM on the concatenated [3C, C]
    weight, then the fused q/k RMSNorm + RoPE; returns (q, k, v) [B,n,H,D] bf16."""
    B, n, _ = x.shape
    W = torch.cat(ws, 0)
    b = torch.cat(bs, 0) if all(t is not None for t in bs) else None
    qkv = _LinearFn.apply(x, W, b, None)
    out = _QKNormRopeFn.apply(qkv, wq_norm, wk_norm, pos, freqs, num_heads, eps)
    C = out.shape[-1] // 3
    D = C // num_heads
    q, k, v = out.split(C, dim=-1)
    return q.reshape(B, n, num_heads, D), k.reshape(B, n, num_heads, D), v.reshape(B, n, num_heads, D)


def linear(x, w, b=None, act: Optional[str] = None):
    if not x.is_cuda:
        y = F.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype))
        return F.gelu(y, approximate="tanh") if act == "gelu_tanh" else y
    if _fused(x, w, b):
        return ops.linear(x, w, b, act)
    return _LinearFn.apply(x, w, b, act)


def gated_residual_linear(x, w, b, resid, gate=None):
    """resid + (x·Wᵀ + b)·gate  (gate [B,C] or None)."""
    if not x.is_cuda:
        y = F.linear(x, w.to(x.dtype), None if b is None else b.to(x.dtype))
        return resid + (y * gate[:, None, :] if gate is not None else y)
    if _fused(x, w, b, resid, gate):
        # in place on the fp32 residual: each output row is read and written by one thread
        out = resid if (resid.dtype == torch.float32 and resid.is_contiguous()) else None
        return ops.linear_gated_residual(x, w, b, resid, gate, out=out)
    y = _LinearFn.apply(x, w, b, None)
    if resid.dtype == torch.float32 and resid.dim() == 3 and y.shape[-1] % 4 == 0:
        return _GatedAddFn.apply(resid, y, gate)
    y = y.float()
    return resid.float() + (y * gate.float()[:, None, :] if gate is not None else y)


def gated_add(resid, y, gate=None):
    """resid + y·gate[b] for a branch output y produced outside the fused GEMM epilogue
    (LoRA / HiF8 projections): the fused forward/backward kernels on CUDA."""
    if (not resid.is_cuda or resid.dtype != torch.float32 or resid.dim() != 3 or y.shape[-1] % 4
            or y.shape != resid.shape):
        return resid + (y * gate[:, None, :] if gate is not None else y)
    if _fused(resid, y, gate):
        return ops.gated_add(resid, y, gate)
    return _GatedAddFn.apply(resid, y.to(_BF16), gate)


# ----------------------------------------------------------------------------- norms

def ln_modulate(x, shift, scale, eps):
    if not x.is_cuda:
        y = F.layer_norm(x.float(), (x.shape[-1],), eps=eps).type_as(x)
        return y * (1 + scale[:, None, :]) + shift[:, None, :]
    if _fused(x, shift, scale):
        return ops.ln_modulate(x, shift, scale, eps)
    if x.dtype == torch.float32 and x.dim() == 3 and x.shape[-1] % 4 == 0 and x.shape[-1] <= 8192:
        return _LNModFn.apply(x.contiguous(), shift.float(), scale.float(), eps)
    y = F.layer_norm(x.float(), (x.shape[-1],), eps=eps)
    return (y * (1 + scale.float()[:, None, :]) + shift.float()[:, None, :]).to(_BF16)


class _AffineLNFn(torch.autograd.Function):
    """bf16 affine LayerNorm of the fp32 residual on the fused kernels: the backward is the
    LN-modulate backward with (1 + scale) = w for every batch entry (dw = Σ dscale,
    db = Σ dshift)."""

    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        ctx.save_for_backward(x, weight)
        ctx.eps = eps
        ctx.has_b = bias is not None
        return ops.layer_norm(x, weight, bias, eps)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        scale = (w.float() - 1.0).expand(x.shape[0], -1)
        dx, dsc, dsh = ops.ln_modulate_bwd(x, dy, scale, ctx.eps)
        return dx, dsc.sum(0).to(w.dtype), (dsh.sum(0) if ctx.has_b else None), None


def layer_norm(x, weight, bias, eps):
    if not x.is_cuda:
        return F.layer_norm(x.float(), (x.shape[-1],), weight, bias, eps).type_as(x)
    if _fused(x, weight, bias):
        return ops.layer_norm(x, weight, bias, eps)
    if (weight is not None and x.dtype == torch.float32 and x.dim() == 3 and x.shape[-1] % 4 == 0
            and x.shape[-1] <= 8192):
        return _AffineLNFn.apply(x.contiguous(), weight, bias, eps)
    w = weight.float() if weight is not None else None
    b = bias.float() if bias is not None else None
    return F.layer_norm(x.float(), (x.shape[-1],), w, b, eps).to(_BF16)


class _RMSNormFn(torch.autograd.Function):
    """bf16 full-row RMSNorm with an fp32 weight, fused forward and backward kernels."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        xb = x.to(_BF16).contiguous()
        ctx.save_for_backward(xb, weight)
        ctx.eps = eps
        ctx.x_dtype = x.dtype
        return ops.rms_norm(xb, weight, eps)

    @staticmethod
    def backward(ctx, dy):
        xb, w = ctx.saved_tensors
        dx, dw = ops.rms_norm_bwd(xb, dy, w, ctx.eps)
        return dx.to(ctx.x_dtype), (dw.to(w.dtype) if w is not None else None), None


def rms_norm(x, weight, eps):
    if not x.is_cuda:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).type_as(x) * weight
    if _fused(x, weight):
        return ops.rms_norm(x, weight, eps)
    if x.shape[-1] % 4 == 0 and x.shape[-1] <= 8192:
        return _RMSNormFn.apply(x, weight, eps)
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * weight.float()


def qk_norm_rope_packed(qkv, wq, wk, pos, freqs, num_heads: int, eps: float):
    """q/k RMSNorm + RoPE on a [B, n, 3C] qkv from any projection (plain, LoRA or HiF8
    Linears): the fused kernel in place without autograd, else the kernel-backed autograd
    function.  Returns (q, k, v) [B, n, H, D]."""
    B, n, C3 = qkv.shape
    C = C3 // 3
    D = C // num_heads
    if _fused(qkv, wq, wk):
        return ops.qk_norm_rope(qkv.to(_BF16).contiguous(), wq, wk, pos, freqs, num_heads, eps)
    out = _QKNormRopeFn.apply(qkv.to(_BF16), wq, wk, pos, freqs, num_heads, eps)
    q, k, v = out.split(C, dim=-1)
    return q.reshape(B, n, num_heads, D), k.reshape(B, n, num_heads, D), v.reshape(B, n, num_heads, D)


def apply_rope(x, pos, freqs):
    """x [B,n,H,D] → rotated fp32 (CPU / autograd path)."""
    return ref.apply_rope(x, pos, freqs)


# ----------------------------------------------------------------------------- attention

class _AttnFn(torch.autograd.Function):
    """Segmented attention with both passes on the tcgen05 kernels: the forward keeps
    (q, k, v, o, LSE) in bf16/fp32, the backward recomputes P from the LSE."""

    @staticmethod
    def forward(ctx, q, k, v, seg_q, seg_k, scale):
        qb, kb, vb = q.to(_BF16), k.to(_BF16), v.to(_BF16)
        o, lse = ops.attention(qb, kb, vb, seg_q, seg_k, scale, return_lse=True)
        ctx.save_for_backward(qb, kb, vb, o, lse)
        ctx.segs = (seg_q, seg_k)
        ctx.scale = scale
        ctx.dtypes = (q.dtype, k.dtype, v.dtype)
        return o

    @staticmethod
    def backward(ctx, go):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = ops.attention_bwd(q, k, v, o, go, lse, ctx.segs[0], ctx.segs[1], ctx.scale)
        tq, tk, tv = ctx.dtypes
        return dq.to(tq), dk.to(tk), dv.to(tv), None, None, None


def attention(q, k, v, seg_q, seg_k, scale=None):
    """Attention inside segments; q [B,nq,H,D], k/v [B,nk,H,D] → [B,nq,H,D]."""
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if not q.is_cuda:
        B, nq, H, _ = q.shape
        outs = []
        sq, sk = seg_q.tolist(), seg_k.tolist()
        for s in range(len(sq) - 1):
            qs = q[:, sq[s]:sq[s + 1]].transpose(1, 2)
            ks = k[:, sk[s]:sk[s + 1]].transpose(1, 2)
            vs = v[:, sk[s]:sk[s + 1]].transpose(1, 2)
            outs.append(F.scaled_dot_product_attention(qs, ks, vs, scale=scale).transpose(1, 2))
        return torch.cat(outs, dim=1)
    if _fused(q, k, v):
        return ops.attention(q, k, v, seg_q, seg_k, scale)
    return _AttnFn.apply(q, k, v, seg_q, seg_k, scale)
