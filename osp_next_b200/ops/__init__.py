"""Fused ops of the OSP-Next DiT.

Every op has one CUDA implementation (hand-written sm_100a kernels in
``ops/csrc``, loaded from the in-tree ``_C.so``) and a PyTorch reference used for
CPU tensors and as the numerics oracle in tests (:mod:`.reference`).  There is
no silent fallback on CUDA tensors: a missing extension raises.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import reference as ref
from ._ext import ext, available  # noqa: F401

_BF16 = torch.bfloat16


def _cuda(*ts) -> bool:
    return any(t is not None and t.is_cuda for t in ts)


def _c(t):
    return t if t is None or t.is_contiguous() else t.contiguous()


# ----------------------------------------------------------------------------- norms

def ln_modulate(x, shift, scale, eps: float = 1e-6):
    """bf16 ``LN(x)·(1+scale)+shift`` (x fp32/bf16 [B,n,C], shift/scale [B,C])."""
    if not _cuda(x):
        return ref.ln_modulate(x, shift, scale, eps)
    x = _c(x)
    out = torch.empty(x.shape, dtype=_BF16, device=x.device)
    ext().ln_modulate(x, _c(shift.float()), _c(scale.float()), None, None, out, float(eps))
    return out


def layer_norm(x, weight, bias, eps: float = 1e-6):
    """bf16 affine LayerNorm (fp32 math)."""
    if not _cuda(x):
        return ref.layer_norm(x, weight, bias, eps)
    x = _c(x)
    out = torch.empty(x.shape, dtype=_BF16, device=x.device)
    w = weight.float().contiguous() if weight is not None else None
    b = bias.float().contiguous() if bias is not None else None
    ext().ln_modulate(x, None, None, w, b, out, float(eps))
    return out


def rms_norm(x, weight, eps: float = 1e-6):
    """bf16 row RMSNorm over the last dim (the full 5120-wide row for q/k)."""
    if not _cuda(x):
        return ref.rms_norm(x, weight, eps)
    x = _c(x)
    out = torch.empty(x.shape, dtype=_BF16, device=x.device)
    ext().rms_norm(x, weight.float().contiguous() if weight is not None else None, out, float(eps))
    return out


# ----------------------------------------------------------------------------- GEMMs

def _extra_pair(extra, M: int, N: int):
    """Second GEMM operand pair (a2 [M,K2], b2 [N,K2]) as contiguous bf16 with K2 padded to
    a multiple of 8 (zero columns), or None."""
    if extra is None:
        return None
    a2, b2 = extra
    a2 = _c(a2.reshape(M, -1).to(_BF16))
    b2 = _c(b2.to(_BF16))
    if a2.shape[1] % 8:
        pk = 8 - a2.shape[1] % 8
        a2 = torch.nn.functional.pad(a2, (0, pk))
        b2 = torch.nn.functional.pad(b2, (0, pk))
    if b2.shape[0] != N:
        raise ValueError(f"second operand pair: b2 has {b2.shape[0]} rows, the GEMM has N = {N}")
    return a2, b2


def linear(x, weight, bias=None, act: Optional[str] = None, out_dtype=_BF16, extra=None):
    """``act(x·Wᵀ [+ a2·b2ᵀ] + b)`` on the tcgen05 GEMM (bf16 in, fp32 accumulate in TMEM).
    ``extra = (a2, b2)`` adds a second operand pair into the same accumulator (a LoRA
    branch: a2 = x·Aᵀ, b2 = scaling·B)."""
    if not _cuda(x):
        y = ref.linear(x, weight, bias, None, torch.float32)
        if extra is not None:
            y = y + extra[0].reshape(y.shape[:-1] + (-1,)).float() @ extra[1].float().t()
        if act == "gelu_tanh":
            y = torch.nn.functional.gelu(y, approximate="tanh")
        return y.to(out_dtype)
    shp = x.shape
    a = _c(x.reshape(-1, shp[-1]).to(_BF16))
    w = _c(weight.to(_BF16))
    N = w.shape[0]
    # the kernel wants K % 8 == 0 (16-byte TMA rows) and N % 32 == 0: zero-pad otherwise
    # (small LoRA ranks, odd token counts in weight gradients)
    if a.shape[1] % 8:
        pk = 8 - a.shape[1] % 8
        a = torch.nn.functional.pad(a, (0, pk))
        w = torch.nn.functional.pad(w, (0, pk))
    b = None if bias is None else bias.float().contiguous()
    if N % 32:
        pn = 32 - N % 32
        w = torch.nn.functional.pad(w, (0, 0, 0, pn))
        b = None if b is None else torch.nn.functional.pad(b, (0, pn))
    out = torch.empty(a.shape[0], w.shape[0], dtype=out_dtype, device=x.device)
    pair = _extra_pair(extra, a.shape[0], N)
    if pair is None:
        ext().gemm(a, w, b, out, 1 if act == "gelu_tanh" else 0, None, None, None, 0, 0)
    else:
        a2, b2 = pair
        if w.shape[0] != N:
            b2 = torch.nn.functional.pad(b2, (0, 0, 0, w.shape[0] - N))
        ext().gemm_dual(a, w, a2, b2, b, out, 1 if act == "gelu_tanh" else 0, None, None, None, 0, 0)
    if out.shape[1] != N:
        out = out[:, :N].contiguous()
    return out.view(*shp[:-1], N)


def gemm_t(a, b, a_mn: bool, b_mn: bool, out_dtype=torch.float32):
    """``A·Bᵀ`` with A = a (or aᵀ when ``a_mn``: a stored [K, M]) and B = b (or bᵀ when
    ``b_mn``: b stored [K, N]) on the tcgen05 GEMM, reading MN-major operands in place.
    Returns None when the shapes miss the kernel's alignment rules (rows of a multiple of
    8 elements, N a multiple of 32) so the caller can fall back."""
    a, b = _c(a.to(_BF16)), _c(b.to(_BF16))
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if a.shape[1] % 8 or b.shape[1] % 8 or N % 32 or not (a_mn or b_mn):
        return None
    out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    ext().gemm_t(a, b, out, bool(a_mn), bool(b_mn))
    return out


def linear_gated_residual(x, weight, bias, resid, gate=None, dest_row=None, n_out=None, out=None, extra=None):
    """``resid + (x·Wᵀ+b)·gate`` with fp32 residual, optional row remap on store.

    x [B,n,K] bf16, resid [B,n,C] fp32 (may alias ``out`` when no remap),
    gate [B,C] or None.  ``dest_row`` [n] int: row m of each batch entry is stored
    at ``dest_row[m]`` of the [B,n_out,C] output (layout change fused in the store).
    """
    if not _cuda(x):
        if extra is not None:
            y = ref.linear(x, weight, bias, None, torch.float32)
            y = y + extra[0].reshape(y.shape[:-1] + (-1,)).float() @ extra[1].float().t()
            y = y * gate[:, None, :] if gate is not None else y
            o = resid.float() + y
            if dest_row is None:
                return o
            res = torch.zeros(o.shape[0], n_out, o.shape[2], dtype=o.dtype)
            res[:, dest_row.long()] = o
            return res
        return ref.linear_gated_residual(x, weight, bias, resid, gate, dest_row, n_out)
    B, n, K = x.shape
    a = _c(x.reshape(B * n, K).to(_BF16))
    w = _c(weight.to(_BF16))
    C = w.shape[0]
    resid = _c(resid.float())
    if dest_row is None:
        if out is None:
            out = resid
        n_out = n
        dr = None
    else:
        if out is None:
            out = torch.empty(B, n_out, C, dtype=torch.float32, device=x.device)
        dr = dest_row.to(device=x.device, dtype=torch.int32).contiguous()
    pair = _extra_pair(extra, B * n, C)
    bb = None if bias is None else bias.float().contiguous()
    gg = None if gate is None else gate.float().contiguous()
    if pair is None:
        ext().gemm(a, w, bb, out.view(-1, C), 0, resid.view(-1, C), gg, dr, n, n_out)
    else:
        ext().gemm_dual(a, w, pair[0], pair[1], bb, out.view(-1, C), 0, resid.view(-1, C), gg, dr, n, n_out)
    return out


def linear_gated_residual_p2p(x, weight, bias, resid, gate, dest_rank, dest_row, out_ptrs, n_stride: int):
    """Fused SSP exchange: row m of every batch entry b of ``resid + (x·Wᵀ+b)·gate`` is
    stored at row ``b·n_stride + dest_row[m]`` of rank ``dest_rank[m]``'s buffer
    (``out_ptrs`` = device int64 table of the peers' buffer base pointers)."""
    B, n, K = x.shape
    a = _c(x.reshape(B * n, K).to(_BF16))
    w = _c(weight.to(_BF16))
    C = w.shape[0]
    ext().gemm_p2p(a, w, None if bias is None else bias.float().contiguous(), _c(resid.float()).view(-1, C),
                   None if gate is None else gate.float().contiguous(), dest_rank, dest_row, out_ptrs, n,
                   int(n_stride))


# ----------------------------------------------------------------------------- training-only ops
# (CUDA only: the autograd wrappers in models/functional.py call them; CPU training uses
# plain PyTorch autograd)

_ROWS_PER_CTA = 32


def _chunks(n: int) -> int:
    return (n + _ROWS_PER_CTA - 1) // _ROWS_PER_CTA


def linear_gelu_aux(x2, w, b, extra=None):
    """(gelu_tanh(x·Wᵀ [+ a2·b2ᵀ] + b), the pre-activation) both bf16, from one GEMM (FFN-up
    training forward; ``extra`` = a LoRA branch as a second operand pair)."""
    N = w.shape[0]
    out = torch.empty(x2.shape[0], N, dtype=_BF16, device=x2.device)
    aux = torch.empty_like(out)
    pair = _extra_pair(extra, x2.shape[0], N)
    ext().gemm_gelu_aux(_c(x2), _c(w.to(_BF16)), None if b is None else b.float().contiguous(), out, aux,
                        None if pair is None else pair[0], None if pair is None else pair[1])
    return out, aux


def bias_grad(g):
    """Σ over rows of g [M, N] (the bias gradient of a Linear) in fp32, read straight from
    bf16: per-chunk column sums on the GPU, then a sum over the chunks (deterministic)."""
    g2 = g.reshape(-1, g.shape[-1])
    if not _cuda(g2) or g2.shape[-1] % 8:
        return g2.float().sum(0)
    g2 = _c(g2.to(_BF16))
    part = torch.empty((g2.shape[0] + 255) // 256, g2.shape[1], dtype=torch.float32, device=g2.device)
    ext().bias_grad(g2, part)
    return part.sum(0)


def gelu_tanh_bwd(dh, pre):
    dpre = torch.empty_like(pre)
    ext().gelu_tanh_bwd(_c(dh.to(_BF16)), _c(pre), dpre)
    return dpre


def ln_modulate_bwd(x, dy, scale, eps: float = 1e-6):
    """→ (dx fp32, dscale [B,C], dshift [B,C]) for y = LN(x)·(1+scale)+shift, x fp32 [B,n,C]."""
    B, n, C = x.shape
    dx = torch.empty_like(x)
    ps = torch.empty(B, _chunks(n), C, dtype=torch.float32, device=x.device)
    ph = torch.empty_like(ps)
    ext().ln_modulate_bwd(_c(x), _c(dy.to(_BF16)), _c(scale.float()), dx, ps, ph, float(eps))
    return dx, ps.sum(1), ph.sum(1)


def gated_add(resid, y, gate=None):
    """resid + y·gate[b] (fp32 out; resid fp32 [B,n,C], y bf16, gate [B,C] or None)."""
    out = torch.empty(resid.shape, dtype=torch.float32, device=resid.device)
    ext().gated_add_fwd(_c(resid.float()), _c(y.to(_BF16)), None if gate is None else _c(gate.float()), out)
    return out


def gated_add_bwd(dout, y, gate):
    """→ (dy bf16 = dout·gate, dgate [B,C] = Σ_rows dout·y)."""
    B, n, C = dout.shape
    dy = torch.empty(dout.shape, dtype=_BF16, device=dout.device)
    part = torch.empty(B, _chunks(n), C, dtype=torch.float32, device=dout.device)
    ext().gated_add_bwd(_c(dout.float()), _c(y.to(_BF16)), _c(gate.float()), dy, part)
    return dy, part.sum(1)


def rms_norm_bwd(x, dy, weight, eps: float = 1e-6):
    """Gradient of :func:`rms_norm` → (dx bf16 like x, dweight fp32 [C])."""
    C = x.shape[-1]
    x2 = x.reshape(-1, C).to(_BF16).contiguous()
    dy2 = dy.reshape(-1, C).to(_BF16).contiguous()
    dx = torch.empty_like(x2)
    part = torch.empty(_chunks(x2.shape[0]), C, dtype=torch.float32, device=x.device)
    ext().rms_norm_bwd(x2, dy2, weight.float().contiguous() if weight is not None else None, dx, part, float(eps))
    return dx.view(x.shape), part.sum(0)


def qk_norm_rope_bwd(raw, dq, dk, dv, wq, wk, pos, freqs, eps: float = 1e-6):
    """Gradient of :func:`qk_norm_rope` w.r.t. the fused qkv [B,n,3C] and the two norm
    weights; ``raw`` = the pre-norm q|k [B,n,2C] (bf16), dq/dk/dv [B,n,H,D]."""
    B, n, C2 = raw.shape
    C = C2 // 2
    D = dq.shape[-1]
    dqkv = torch.empty(B, n, 3 * C, dtype=_BF16, device=raw.device)
    dqkv[..., 2 * C:] = dv.reshape(B, n, C)
    pos = pos.to(device=raw.device, dtype=torch.int32).contiguous()
    cs = rope_cos_sin(freqs, raw.device)
    dws = []
    for part, (g, w) in enumerate(((dq, wq), (dk, wk))):
        g2 = g.reshape(B * n, C)
        if g2.dtype not in (_BF16, torch.float32):
            g2 = g2.float()
        if g2.stride(-1) != 1 or (g2.stride(0) * g2.element_size()) % 16:
            g2 = g2.contiguous()
        dwp = torch.empty(B, _chunks(n), C, dtype=torch.float32, device=raw.device)
        ext().qk_norm_rope_bwd(raw.reshape(B * n, C2), g2, _c(w.float()), pos, cs, dqkv.view(B * n, 3 * C), dwp,
                               part, B, n, C, D, float(eps))
        dws.append(dwp.sum((0, 1)))
    return dqkv, dws[0], dws[1]


# ----------------------------------------------------------------------------- attention

_CS_CACHE = {}


def rope_cos_sin(freqs: torch.Tensor, device) -> torch.Tensor:
    """(cos, sin) table [L, D/2, 2] fp32 of an angle table, evaluated in fp64 once per
    table (cached), so the kernels rotate with table loads instead of sincos."""
    key = (freqs.data_ptr(), freqs._version, tuple(freqs.shape), str(device))
    hit = _CS_CACHE.get(key)
    if hit is not None and hit[0] is freqs:
        return hit[1]
    a = freqs.to(device=device, dtype=torch.float64)
    cs = torch.stack([a.cos(), a.sin()], -1).float().contiguous()
    if len(_CS_CACHE) > 16:
        _CS_CACHE.clear()
    _CS_CACHE[key] = (freqs, cs)
    return cs


def qk_norm_rope(qkv, wq, wk, pos, freqs, num_heads: int, eps: float = 1e-6):
    """Fused full-row RMSNorm(q), RMSNorm(k) and 3-D RoPE on a fused qkv buffer.

    CUDA: in place on ``qkv`` [B,n,3C] bf16; returns (q,k,v) as strided views
    [B,n,H,D] into it.  ``pos`` int32 [n,3]; ``freqs`` fp32 angle table.
    """
    if not _cuda(qkv):
        return ref.qk_norm_rope(qkv, wq, wk, pos, freqs, num_heads, eps)
    B, n, C3 = qkv.shape
    C = C3 // 3
    D = C // num_heads
    ext().qk_norm_rope(qkv, wq.float().contiguous(), wk.float().contiguous(),
                       pos.to(device=qkv.device, dtype=torch.int32).contiguous(),
                       rope_cos_sin(freqs, qkv.device), num_heads, float(eps))
    q, k, v = qkv.split(C, dim=-1)
    return q.view(B, n, num_heads, D), k.view(B, n, num_heads, D), v.view(B, n, num_heads, D)


_SEG_CACHE = {}


def _seg_dev(seg: torch.Tensor, device):
    """Device copy (int32) and max segment length of a CPU segment table, cached."""
    if seg.is_cuda:
        return seg.to(torch.int32), int((seg[1:] - seg[:-1]).max().item())
    key = (seg.data_ptr(), seg.numel(), str(device))
    hit = _SEG_CACHE.get(key)
    if hit is not None and hit[0] is seg:
        return hit[1], hit[2]
    d = seg.to(device=device, dtype=torch.int32)
    mx = int((seg[1:] - seg[:-1]).max().item()) if seg.numel() > 1 else 0
    if len(_SEG_CACHE) > 256:
        _SEG_CACHE.clear()
    _SEG_CACHE[key] = (seg, d, mx)
    return d, mx


def attention(q, k, v, seg_q, seg_k, scale: Optional[float] = None, return_lse: bool = False):
    """Segmented non-causal attention on the tcgen05 flash kernel.

    q [B,nq,H,D], k/v [B,nk,H,D] (row-strided views allowed; heads packed, last
    dim contiguous).  ``seg_q``/``seg_k`` int32 offsets (CPU tensors preferred:
    the device copy is cached).  Returns o [B,nq,H,D] bf16 contiguous
    (+ LSE [B,H,nq] fp32, natural log).
    """
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if not _cuda(q):
        return ref.attention(q, k, v, seg_q, seg_k, scale, return_lse)
    B, nq, H, _ = q.shape
    out = torch.empty(B, nq, H, D, dtype=_BF16, device=q.device)
    lse = torch.empty(B, H, nq, dtype=torch.float32, device=q.device) if return_lse else torch.empty(0, device=q.device)
    sq, max_q = _seg_dev(seg_q, q.device)
    sk, _ = _seg_dev(seg_k, q.device)
    ext().attention_fwd(q, k, v, sq, sk, out, lse, float(scale), max_q)
    return (out, lse) if return_lse else out


def attention_bwd(q, k, v, o, dout, lse, seg_q, seg_k, scale: Optional[float] = None):
    """Gradients (dq, dk, dv) of :func:`attention` on the tcgen05 backward kernels.

    q [B,nq,H,D], k/v [B,nk,H,D] bf16 (row-strided views allowed), o/dout contiguous
    [B,nq,H,D] bf16, lse [B,H,nq] fp32 from the forward.  Returns contiguous bf16 grads.
    """
    D = q.shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if not _cuda(q):
        return ref.attention_bwd(q, k, v, dout, seg_q, seg_k, scale)
    dq = torch.empty(q.shape, dtype=_BF16, device=q.device)
    dk = torch.empty(k.shape, dtype=_BF16, device=q.device)
    dv = torch.empty(v.shape, dtype=_BF16, device=q.device)
    delta = torch.empty(q.shape[0], q.shape[2], q.shape[1], dtype=torch.float32, device=q.device)
    sq, max_q = _seg_dev(seg_q, q.device)
    sk, max_k = _seg_dev(seg_k, q.device)
    ext().attention_bwd(q, k, v, _c(o.to(_BF16)), _c(dout.to(_BF16)), _c(lse.float()), sq, sk, dq, dk, dv, delta,
                        float(scale), max_q, max_k)
    return dq, dk, dv


def sde_step(x, v, sigma: float, dt: float, sigma_min: float, sigma_max: float, noise=None, prev_sample=None):
    """Fused GRPO SDE step (CUDA) → (prev_sample f32, log_prob [B] f32, mean f32)."""
    x = _c(x.float())
    v = _c(v.float())
    prev = torch.empty_like(x)
    mean = torch.empty_like(x)
    logp = torch.zeros(x.shape[0], dtype=torch.float32, device=x.device)
    ext().sde_step(x, v, None if noise is None else _c(noise.float()),
                   None if prev_sample is None else _c(prev_sample.float()), prev, mean, logp,
                   float(sigma), float(dt), float(sigma_min), float(sigma_max))
    return prev, logp, mean


def adamw_(p, g, m, v, lr, beta1, beta2, eps, weight_decay, step, grad_scale=1.0):
    """In-place fused AdamW on flat fp32 shards (CUDA)."""
    ext().adamw(p, _c(g), m, v, float(lr), float(beta1), float(beta2), float(eps), float(weight_decay), int(step),
                float(grad_scale))


# ----------------------------------------------------------------------------- sampler / quant

def cfg_euler_step(latents, cond, uncond, guidance: float, dt: float):
    if not _cuda(latents):
        return ref.cfg_euler_step(latents, cond, uncond, guidance, dt)
    out = torch.empty_like(latents)
    ext().cfg_euler(_c(latents), _c(cond), _c(uncond), out, float(guidance), float(dt))
    return out


def hif8_round(x):
    if not _cuda(x):
        return ref.hif8_round(x)
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    ext().hif8_round(_c(x.float()), out, 1.0)
    return out


def hif8_quant_dequant(x, scale_max: float = 15.0):
    """Per-tensor scaled HiF8 fake-quant; amax on device, no host sync."""
    if not _cuda(x):
        return ref.hif8_quant_dequant(x, scale_max)
    xc = _c(x)
    out = torch.empty_like(xc)
    ext().hif8_qdq(xc, out, float(scale_max))
    return out


# ----------------------------------------------------------------------------- device errors

ERROR_NAMES = {
    101: "GEMM producer wait", 102: "GEMM MMA wait", 103: "GEMM epilogue wait", 104: "GEMM teardown",
    201: "attention producer wait", 202: "attention MMA wait", 203: "attention softmax wait",
    204: "attention teardown", 205: "attention shared-memory alignment",
    301: "NVLink peer barrier timeout", 302: "NVLink peer barrier slot mismatch",
    901: "probe mbarrier wait", 902: "probe flag wait",
}


class DeviceWaitError(RuntimeError):
    """A bounded wait inside one of the framework's kernels gave up (a peer rank stalled or
    died, or a pipeline stage never arrived).  The kernel skipped its remaining work, so
    the results of the step that raised are not valid."""

    def __init__(self, code: int, device: int, where: str = ""):
        self.code = code
        self.device = device
        name = ERROR_NAMES.get(code, "unknown")
        super().__init__(f"device {device}: kernel error {code} ({name})" + (f" during {where}" if where else ""))


def check_device_errors(device=None, where: str = "") -> None:
    """Read (and clear) the device error word; raise :class:`DeviceWaitError` if it is set.

    One 4-byte device read after a device synchronize: call it at step boundaries (the
    samplers and trainers do) and before writing a checkpoint.  No-op without a GPU."""
    if not torch.cuda.is_available():
        return
    if device is None:
        device = torch.cuda.current_device()
    elif isinstance(device, torch.device):
        if device.type != "cuda":
            return
        device = device.index if device.index is not None else torch.cuda.current_device()
    code = int(ext().get_error(int(device), True))
    if code:
        raise DeviceWaitError(code, int(device), where)


def check_device_errors_all_ranks(device, where: str = "", group=None) -> None:
    """:func:`check_device_errors` agreed over the process group: every rank raises if any
    rank's kernels recorded an error, so all ranks stop at the same step boundary."""
    import torch.distributed as dist
    code = 0
    dev_index = None
    if torch.cuda.is_available() and (not isinstance(device, torch.device) or device.type == "cuda"):
        dev_index = device.index if isinstance(device, torch.device) else int(device)
        if dev_index is None:
            dev_index = torch.cuda.current_device()
        code = int(ext().get_error(dev_index, True))
    if dist.is_available() and dist.is_initialized():
        t = torch.tensor([code], dtype=torch.int64,
                         device=torch.device("cuda", dev_index) if dev_index is not None else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        code = int(t.item())
    if code:
        raise DeviceWaitError(code, -1 if dev_index is None else dev_index, (where + " (some rank)").strip())
