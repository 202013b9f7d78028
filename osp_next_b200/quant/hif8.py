"""HiF8 fake quantisation: linear layers, attention inputs, and the quantiser API.

Reference: ospnext/modules/hif8_linear.py:42-170 and hif8_attention.py:40-127
(per-tensor dynamic scale ``s = scale_max / max(|x|, 1e-8)``, quantise→dequantise
x and W in forward, the incoming gradient in backward, straight-through
estimator; q/k/v quantised before attention and dq/dk/dv after), plus the
``quant_cy_npu`` surface those files import (QTensor.quant_dequant_float,
QType, QLinear, replace_linear).  The reference can only run this on Ascend
NPUs; here the rounding is the sm_100a kernel in ops/csrc/misc.cu (same grid as
the Ascend kernel) and the matmuls are the tcgen05 GEMM.  GEMMs stay bf16: the
reference emulates HiF8, it has no 8-bit matmul.
"""
from __future__ import annotations

from copy import deepcopy
from typing import List, Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..ops import reference as ref


def _out_dtype(dt: torch.dtype) -> torch.dtype:
    """GEMM output dtype for a gradient whose tensor has dtype ``dt``: bf16 stays bf16
    (rounded once from the fp32 accumulator), anything else is produced in fp32."""
    return torch.bfloat16 if dt == torch.bfloat16 else torch.float32


def quant(x: torch.Tensor, scale_max: float) -> torch.Tensor:
    """Scaled HiF8 quantise→dequantise of a whole tensor (device amax, no host sync)."""
    if x.is_cuda:
        return ops.hif8_quant_dequant(x.contiguous(), scale_max)
    return ref.hif8_quant_dequant(x, scale_max)


class _HIF8LinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, smf: float, smb: float):
        x_q = quant(x, smf)
        w_q = quant(weight, smf)
        ctx.save_for_backward(x_q, w_q)
        ctx.smb = smb
        ctx.has_bias = bias is not None
        if x.is_cuda:
            return ops.linear(x_q.reshape(-1, x.shape[-1]), w_q, bias).view(*x.shape[:-1], weight.shape[0])
        return F.linear(x_q, w_q, bias)

    @staticmethod
    def backward(ctx, g):
        x_q, w_q = ctx.saved_tensors
        g_q = quant(g, ctx.smb)
        g2 = g_q.reshape(-1, g_q.shape[-1])
        x2 = x_q.reshape(-1, x_q.shape[-1])
        if g.is_cuda:
            gb = g2.to(torch.bfloat16)
            wb, xb = w_q.to(torch.bfloat16), x2.to(torch.bfloat16)
            # operands read MN-major in place; transposed copies only where the shapes miss
            # the kernel's alignment rules
            # bf16 inputs / weights take their gradients in bf16 straight from the GEMM
            # epilogue (fp32 accumulation rounded once, as the conversion would)
            dx = ops.gemm_t(gb, wb, a_mn=False, b_mn=True, out_dtype=_out_dtype(x_q.dtype))
            if dx is None:
                dx = ops.linear(gb, wb.t().contiguous(), None, out_dtype=torch.float32)
            dw = ops.gemm_t(gb, xb, a_mn=True, b_mn=True, out_dtype=_out_dtype(w_q.dtype))
            if dw is None:
                dw = ops.linear(gb.t().contiguous(), xb.t().contiguous(), None, out_dtype=torch.float32)
            db = ops.bias_grad(gb) if ctx.has_bias else None
        else:
            dx = g2 @ w_q
            dw = g2.t() @ x2
            db = g2.float().sum(0) if ctx.has_bias else None
        return dx.view(x_q.shape).to(x_q.dtype), dw.to(w_q.dtype), db, None, None


class _HIF8MultiLinearFn(torch.autograd.Function):
    """Several HiF8 Linears that read the same input (q/k/v, or one Linear with a GELU
    epilogue): x is quantised once, each weight with its own per-tensor scale, and one
    GEMM runs on the concatenated quantised weights.  Backward quantises each output
    slice's gradient with its own scale (exactly what separate HIF8Linear modules do) and
    runs dX and dW as one GEMM each over the packed slices.  CUDA only."""

    @staticmethod
    def forward(ctx, x, smf, smb, act, n, *wb):
        ws, bs = wb[:n], wb[n:]
        x_q = quant(x.to(torch.bfloat16).contiguous(), smf)
        # each weight quantised in its own dtype, as HIF8Linear does, then bf16 for the GEMM
        w_q = torch.cat([quant(w.detach().contiguous(), smf).to(torch.bfloat16) for w in ws], 0)
        has_b = all(b is not None for b in bs)
        b = torch.cat([b_.float() for b_ in bs], 0) if has_b else None
        x2 = x_q.reshape(-1, x.shape[-1])
        pre = None
        if act == "gelu_tanh" and w_q.shape[0] % 32 == 0 and x2.shape[1] % 8 == 0:
            y, pre = ops.linear_gelu_aux(x2, w_q, b)
        elif act == "gelu_tanh":
            pre = ops.linear(x2, w_q, b, None)
            y = F.gelu(pre.float(), approximate="tanh").to(torch.bfloat16)
        else:
            y = ops.linear(x2, w_q, b, None)
        ctx.save_for_backward(x_q, w_q, pre)
        ctx.meta = (smb, act, [w.shape[0] for w in ws], [w.dtype for w in ws], has_b, x.dtype, x.shape)
        return y.view(*x.shape[:-1], w_q.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x_q, w_q, pre = ctx.saved_tensors
        smb, act, outs, wdts, has_b, xdt, xshape = ctx.meta
        g = gy.reshape(-1, gy.shape[-1])
        if act == "gelu_tanh":
            g = ops.gelu_tanh_bwd(g, pre.to(torch.bfloat16)) if pre.dtype == torch.bfloat16 else \
                torch.autograd.grad(F.gelu(pre.float().requires_grad_(True), approximate="tanh"), pre, g.float())[0]
        # per-slice gradient quantisation (one scale per original Linear)
        parts, o = [], 0
        for n_out in outs:
            parts.append(quant(g[:, o:o + n_out].contiguous().to(torch.bfloat16), smb))
            o += n_out
        gq = torch.cat(parts, 1) if len(parts) > 1 else parts[0]
        x2 = x_q.reshape(-1, x_q.shape[-1])
        dx = ops.gemm_t(gq, w_q, a_mn=False, b_mn=True, out_dtype=_out_dtype(xdt))
        if dx is None:
            dx = ops.linear(gq, w_q.t().contiguous(), None, out_dtype=torch.float32)
        w_out = torch.bfloat16 if all(t == torch.bfloat16 for t in wdts) else torch.float32
        dw = ops.gemm_t(gq, x2, a_mn=True, b_mn=True, out_dtype=w_out)
        if dw is None:
            dw = ops.linear(gq.t().contiguous(), x2.t().contiguous(), None, out_dtype=torch.float32)
        dws = list(dw.split(outs, 0))
        dbs = list(ops.bias_grad(gq).split(outs, 0)) if has_b else [None] * len(outs)
        grads = [dx.view(xshape).to(xdt), None, None, None, None]
        grads += [d.to(t) for d, t in zip(dws, wdts)] + dbs
        return tuple(grads)


def hif8_multi_linear(x, linears, act=None):
    """y = [HIF8Linear_1(x) | … | HIF8Linear_n(x)] (optionally gelu_tanh of it) in one GEMM,
    with the same quantisation semantics as calling each module.  ``linears`` share one
    input and the scale settings of the first."""
    l0 = linears[0]
    smf, smb = l0.scale_max_forward, l0.scale_max_backward
    if not x.is_cuda:
        y = torch.cat([m(x) for m in linears], -1)
        return F.gelu(y, approximate="tanh") if act == "gelu_tanh" else y
    if not (torch.is_grad_enabled() and (x.requires_grad or any(m.weight.requires_grad for m in linears))):
        x_q = quant(x.to(torch.bfloat16).contiguous(), smf)
        if len(linears) == 1:
            w_q = l0._cached_wq()
        else:                        # packed quantised weights, rebuilt when any weight changes
            key = tuple((m.weight.data_ptr(), m.weight._version) for m in linears)
            hit = getattr(l0, "_packed_wq", None)
            if hit is None or hit[0] != key:
                hit = (key, torch.cat([m._cached_wq() for m in linears], 0))
                l0._packed_wq = hit
            w_q = hit[1]
        bs = [m.bias for m in linears]
        b = torch.cat([b_.float() for b_ in bs], 0) if all(b_ is not None for b_ in bs) else None
        y = ops.linear(x_q.reshape(-1, x.shape[-1]), w_q, b, act)
        return y.view(*x.shape[:-1], w_q.shape[0])
    ws = [m.weight for m in linears]
    bs = [m.bias for m in linears]
    return _HIF8MultiLinearFn.apply(x, smf, smb, act, len(linears), *ws, *bs)


class HIF8Linear(nn.Linear):
    """Drop-in ``nn.Linear`` with HiF8 fake quantisation of x, W (forward) and dY (backward)."""
    is_hif8 = True

    def __init__(self, in_features, out_features, bias=True, scale_max_forward=15.0, scale_max_backward=224.0,
                 device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device=device, dtype=dtype)
        self.scale_max_forward = scale_max_forward
        self.scale_max_backward = scale_max_backward
        self._wq = None

    def _cached_wq(self):
        key = (self.weight.data_ptr(), self.weight._version)
        if self._wq is None or self._wq[0] != key:
            self._wq = (key, quant(self.weight.detach(), self.scale_max_forward).to(torch.bfloat16))
        return self._wq[1]

    def forward(self, x):
        if x.is_cuda and not (torch.is_grad_enabled() and (x.requires_grad or self.weight.requires_grad)):
            x_q = quant(x.to(torch.bfloat16), self.scale_max_forward)
            return ops.linear(x_q.reshape(-1, x.shape[-1]), self._cached_wq(), self.bias).view(
                *x.shape[:-1], self.out_features)
        return _HIF8LinearFunction.apply(x, self.weight, self.bias, self.scale_max_forward, self.scale_max_backward)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}, "
                f"scale_max_fwd={self.scale_max_forward}, scale_max_bwd={self.scale_max_backward}")


class _HIF8QKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, smf, smb):
        ctx.smb = smb
        return quant(q, smf), quant(k, smf), quant(v, smf)

    @staticmethod
    def backward(ctx, gq, gk, gv):
        f = (lambda g: None if g is None else quant(g.contiguous(), ctx.smb))
        return f(gq), f(gk), f(gv), None, None


def hif8_qkv(q, k, v, scale_max_forward=15.0, scale_max_backward=224.0):
    """Quantise q/k/v (forward) and dq/dk/dv (backward) around any attention call."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        return _HIF8QKV.apply(q, k, v, scale_max_forward, scale_max_backward)
    return quant(q, scale_max_forward), quant(k, scale_max_forward), quant(v, scale_max_forward)


# ----------------------------------------------------------------------------- quantiser API

class QType:
    """Quantisation format descriptor (subset of quant_cy_npu/base/QType.py used by OSP-Next)."""

    def __init__(self, desc: str):
        if desc not in ("hif8", "bf16", "fp16", "fp32"):
            raise ValueError(f"unsupported QType {desc!r}")
        self.desc = desc
        self.q_dim = -1

    def dim(self, d):
        out = deepcopy(self)
        out.q_dim = d
        return out

    def dim_(self, d):
        self.q_dim = d
        return self

    def copy(self):
        return deepcopy(self)

    def __repr__(self):
        return f"QType: {self.desc}   Dim: {self.q_dim}"


def quant_dequant_float(x: torch.Tensor, qtype: Union[QType, str], force_fp32: bool = False) -> torch.Tensor:
    """Round ``x`` (already scaled) to the format's grid (QTensor.py:94-128 semantics)."""
    desc = qtype if isinstance(qtype, str) else qtype.desc
    if desc == "hif8":
        y = ops.hif8_round(x.float().contiguous()) if x.is_cuda else ref.hif8_round(x)
    elif desc == "bf16":
        y = x.to(torch.bfloat16).float()
    elif desc == "fp16":
        y = x.to(torch.float16).float()
    else:
        y = x.float()
    return y if force_fp32 else y.to(x.dtype)


def quant_hif8(x: torch.Tensor) -> torch.Tensor:
    """The reference's PyTorch formula (QFuncs/hif8.py:7-23), kept as a second oracle."""
    return ref.hif8_round_torch_oracle(x)


class QLinear(nn.Linear):
    """Linear with fake-quantised weight / input / gradient (QLinear.py semantics, HiF8 grids)."""

    def __init__(self, in_features, out_features, bias=True):
        super().__init__(in_features, out_features, bias)
        self.w_qtype: Optional[QType] = None
        self.in_qtype: Optional[QType] = None
        self.quant_grad = True

    def transfer(self, m: nn.Linear):
        with torch.no_grad():
            self.weight.copy_(m.weight)
            if m.bias is not None:
                self.bias.copy_(m.bias)

    def assign_qparams(self, q):
        self.w_qtype = QType(q) if isinstance(q, str) else q

    def assign_input_qparams(self, q):
        self.in_qtype = QType(q) if isinstance(q, str) else q

    def set_quant_grad(self, flag: bool):
        self.quant_grad = flag

    def forward(self, x):
        w = quant_dequant_float(self.weight, self.w_qtype, True).to(x.dtype) if self.w_qtype else self.weight
        xi = quant_dequant_float(x, self.in_qtype, True).to(x.dtype) if self.in_qtype else x
        # straight-through: forward uses the rounded values, gradients pass unchanged
        w = self.weight + (w - self.weight).detach()
        xi = x + (xi - x).detach()
        return F.linear(xi, w, self.bias)


def replace_linear(module: nn.Module, w_Q, in_Q=None, quant_grad: bool = True, exclude_layers: List[str] = ()):
    """Swap every ``nn.Linear`` of ``module`` for a :class:`QLinear` (utils/utils.py:16-40)."""
    mods = dict(module.named_modules())
    for n, m in list(module.named_modules()):
        if n in exclude_layers or type(m) is not nn.Linear:
            continue
        q = QLinear(m.in_features, m.out_features, m.bias is not None).to(m.weight.device, m.weight.dtype)
        q.transfer(m)
        q.assign_qparams(w_Q)
        q.set_quant_grad(quant_grad)
        if in_Q is not None:
            q.assign_input_qparams(in_Q)
        parent = mods[".".join(n.split(".")[:-1])]
        setattr(parent, n.split(".")[-1], q)
    return module
