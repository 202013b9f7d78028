"""PyTorch reference math for every fused op (fp32 internally).

These functions define the numerics the sm_100a kernels must match and are the
code path for CPU tensors (unit tests, Gloo multi-process tests).  Each states
the reference expression it reproduces.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F


def ln_modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, eps: float = 1e-6,
                out_dtype=torch.bfloat16) -> torch.Tensor:
    """``LN(x)·(1+scale)+shift`` with a non-affine LayerNorm in fp32
    (osp_next.py:941, 954; want2v.py:96-106).  x [B,n,C]; shift/scale [B,C]."""
    xf = x.float()
    y = F.layer_norm(xf, (xf.shape[-1],), eps=eps)
    y = y * (1.0 + scale.float()[:, None, :]) + shift.float()[:, None, :]
    return y.to(out_dtype)


def layer_norm(x: torch.Tensor, weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
               eps: float = 1e-6, out_dtype=torch.bfloat16) -> torch.Tensor:
    """Affine LayerNorm in fp32 (norm3, osp_next.py:949-953)."""
    xf = x.float()
    w = weight.float() if weight is not None else None
    b = bias.float() if bias is not None else None
    return F.layer_norm(xf, (xf.shape[-1],), w, b, eps).to(out_dtype)


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float = 1e-6,
             out_dtype=torch.bfloat16) -> torch.Tensor:
    """Row RMSNorm over the full last dim (WanRMSNorm, want2v.py:77-93)."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(out_dtype)


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           act: Optional[str] = None, out_dtype=torch.bfloat16) -> torch.Tensor:
    """``act(x·Wᵀ + b)``; bf16 operands, fp32 accumulation (nn.Linear under bf16 autocast)."""
    y = x.to(torch.bfloat16).float() @ weight.to(torch.bfloat16).float().t()
    if bias is not None:
        y = y + bias.float()
    if act == "gelu_tanh":
        y = gelu_tanh(y)
    elif act is not None:
        raise ValueError(act)
    return y.to(out_dtype)


def linear_gated_residual(x, weight, bias, resid, gate=None, dest_row=None, n_out=None):
    """``out = resid + (x·Wᵀ + b)·gate`` (osp_next.py:947, 956), fp32 residual.

    x [B,n,K] bf16, resid [B,n,C] fp32, gate [B,C] (None → 1).  With
    ``dest_row`` the result row m of every batch entry is stored at row
    ``dest_row[m]`` of a fresh [B,n_out,C] tensor (layout change fused in the store).
    """
    y = x.to(torch.bfloat16).float() @ weight.to(torch.bfloat16).float().t()
    if bias is not None:
        y = y + bias.float()
    y = y.to(torch.bfloat16).float()            # Linear output is bf16 under autocast
    if gate is not None:
        y = y * gate.float()[:, None, :]
    out = resid.float() + y
    if dest_row is None:
        return out
    o = out.new_zeros(out.shape[0], n_out, out.shape[2])
    o[:, dest_row.to(out.device)] = out
    return o


def rope_freqs(head_dim: int, max_len: int = 1024, theta: float = 10000.0) -> torch.Tensor:
    """Angle table [max_len, head_dim/2] (fp32 from fp64), split t|h|w.

    osp_next.py:63-70, 1237-1246: ``rope_params(1024, D-4⌊D/6⌋) ‖ rope_params(1024, 2⌊D/6⌋) ×2``.
    """
    def params(dim):
        return torch.outer(torch.arange(max_len, dtype=torch.float64),
                           1.0 / torch.pow(theta, torch.arange(0, dim, 2, dtype=torch.float64).div(dim))).float()
    d = head_dim
    return torch.cat([params(d - 4 * (d // 6)), params(2 * (d // 6)), params(2 * (d // 6))], dim=1)


def rope_split(head_dim: int):
    c = head_dim // 2
    return c - 2 * (c // 3), c // 3, c // 3


def rope_angles(pos: torch.Tensor, freqs: torch.Tensor, head_dim: int) -> torch.Tensor:
    """Angles [n, D/2] for positions pos [n,3] (t,h,w)."""
    ct, ch, cw = rope_split(head_dim)
    ft, fh, fw = freqs.split([ct, ch, cw], dim=1)
    p = pos.long().to(freqs.device)
    return torch.cat([ft[p[:, 0]], fh[p[:, 1]], fw[p[:, 2]]], dim=1)


def apply_rope(x: torch.Tensor, pos: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair complex rotation in fp32 (osp_next.py:608-644). x [B,n,H,D]."""
    B, n, H, D = x.shape
    ang = rope_angles(pos, freqs, D)                       # [n, D/2]
    cos = ang.cos()[None, :, None, :]
    sin = ang.sin()[None, :, None, :]
    xf = x.float().reshape(B, n, H, D // 2, 2)
    x1, x2 = xf[..., 0], xf[..., 1]
    o1 = x1 * cos - x2 * sin
    o2 = x1 * sin + x2 * cos
    return torch.stack([o1, o2], dim=-1).flatten(3)


def qk_norm_rope(qkv: torch.Tensor, wq, wk, pos: torch.Tensor, freqs: torch.Tensor,
                 num_heads: int, eps: float = 1e-6):
    """Split fused qkv [B,n,3C] → (q,k,v) bf16 [B,n,H,D] with full-row RMSNorm on q,k
    and 3-D RoPE (osp_next.py:742-752)."""
    B, n, C3 = qkv.shape
    C = C3 // 3
    D = C // num_heads
    q, k, v = qkv.split(C, dim=-1)
    q = rms_norm(q, wq, eps, torch.float32).view(B, n, num_heads, D)
    k = rms_norm(k, wk, eps, torch.float32).view(B, n, num_heads, D)
    q = apply_rope(q, pos, freqs).to(torch.bfloat16)
    k = apply_rope(k, pos, freqs).to(torch.bfloat16)
    return q, k, v.reshape(B, n, num_heads, D).to(torch.bfloat16)


def attention(q, k, v, seg_q: torch.Tensor, seg_k: torch.Tensor, scale: Optional[float] = None,
              return_lse: bool = False):
    """Non-causal softmax attention inside segments.

    q [B,nq,H,D], k/v [B,nk,H,D]; segment s pairs q rows seg_q[s]:seg_q[s+1] with
    k rows seg_k[s]:seg_k[s+1] (a Skiparse group, or all rows).  Output
    [B,nq,H,D] bf16 (+ LSE [B,H,nq] fp32, natural log).
    """
    B, nq, H, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    out = torch.empty(B, nq, H, D, dtype=torch.float32, device=q.device)
    lse = torch.empty(B, H, nq, dtype=torch.float32, device=q.device)
    sq = seg_q.tolist()
    sk = seg_k.tolist()
    for s in range(len(sq) - 1):
        qs = q[:, sq[s]:sq[s + 1]].float().transpose(1, 2)       # B,H,L,D
        ks = k[:, sk[s]:sk[s + 1]].float().transpose(1, 2)
        vs = v[:, sk[s]:sk[s + 1]].float().transpose(1, 2)
        logits = (qs @ ks.transpose(-1, -2)) * scale
        l = torch.logsumexp(logits, dim=-1)
        p = torch.exp(logits - l[..., None])
        out[:, sq[s]:sq[s + 1]] = (p @ vs).transpose(1, 2)
        lse[:, :, sq[s]:sq[s + 1]] = l
    o = out.to(torch.bfloat16)
    return (o, lse) if return_lse else o


def attention_bwd(q, k, v, dout, seg_q: torch.Tensor, seg_k: torch.Tensor, scale: Optional[float] = None):
    """fp32 gradients (dq, dk, dv) of :func:`attention` by autograd of the same math."""
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    sq, sk = seg_q.tolist(), seg_k.tolist()
    outs = []
    for s in range(len(sq) - 1):
        qs = qf[:, sq[s]:sq[s + 1]].transpose(1, 2)
        ks = kf[:, sk[s]:sk[s + 1]].transpose(1, 2)
        vs = vf[:, sk[s]:sk[s + 1]].transpose(1, 2)
        p = torch.softmax((qs @ ks.transpose(-1, -2)) * scale, dim=-1)
        outs.append((p @ vs).transpose(1, 2))
    o = torch.cat(outs, dim=1)
    o.backward(dout.float())
    return qf.grad, kf.grad, vf.grad


def cfg_euler_step(latents, cond, uncond, guidance: float, dt: float):
    """``x + (u + g·(c−u))·dt`` in fp32, cast back (flow_matching.py:116-127, 178-184)."""
    v = uncond.float() + guidance * (cond.float() - uncond.float())
    return (latents.float() + v * dt).to(latents.dtype)


def hif8_quant_dequant(x: torch.Tensor, scale_max: float = 15.0) -> torch.Tensor:
    """Per-tensor dynamic-scale HiF8 fake quantization (kernel semantics).

    ``s = scale_max / amax(|x|)`` (as torch evaluates it: 1/amax, then times scale_max);
    y = Q(x·s)/s where Q rounds to the HiF8 grid as
    the Ascend kernel does (quant_cy_npu/base/cusrc/hif8_quant_op.h:88-151):
    exponent e from the fp32 bits; mantissa bits 3/2/1/0 for |e| ≤ 3/7/15/else;
    step ``2^(max(e,−22) − m)``; round half away from zero; |v| < 2⁻²³ → 0;
    |v| ≥ 40960 → ±inf.  See :func:`hif8_round` for the grid alone.
    """
    amax = x.detach().abs().max().float().clamp(min=1e-8)
    s = amax.reciprocal() * scale_max      # what torch makes of `scale_max / amax` (hif8_linear.py:46)
    y = hif8_round(x.float() * s) / s
    return y.to(x.dtype)


def hif8_round(v: torch.Tensor) -> torch.Tensor:
    """Round fp32 values to the HiF8 grid (kernel semantics, see above)."""
    v = v.float()
    a = v.abs()
    bits = a.view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 127                     # exact exponent from the bits
    ae = e.abs()
    m = torch.where(ae <= 3, 3, torch.where(ae <= 7, 2, torch.where(ae <= 15, 1, 0)))
    step_exp = torch.clamp(e, min=-22) - m
    step = torch.pow(torch.tensor(2.0, dtype=torch.float32), step_exp.float())
    q = torch.floor(a / step + 0.5) * step
    q = torch.where(a < 2.0 ** -23, torch.zeros_like(q), q)
    q = torch.where(a >= 40960.0, torch.full_like(q, float("inf")), q)
    return torch.copysign(q, v)


def hif8_round_torch_oracle(x: torch.Tensor) -> torch.Tensor:
    """The reference's PyTorch formula (quant_cy_npu/base/QFuncs/hif8.py:7-23):
    exponent from fp32 ``log2``, no floor, no saturation."""
    x = x.float()
    e = torch.floor(torch.log2(x.abs() + 2.0 ** -45))
    ae = e.abs()
    m = torch.where(ae <= 3, 3.0, torch.where(ae <= 7, 2.0, torch.where(ae <= 15, 1.0, 0.0)))
    return torch.sign(x) * torch.floor(x.abs() * torch.pow(2.0, m - e) + 0.5) * torch.pow(2.0, e - m)
