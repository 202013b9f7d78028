"""Remaining quant_cy_npu surface: sparse / quantised Linear and Conv layers and the
block-floating-point quantiser (reference: ospnext/quant_cy_npu/layers/SLinear.py,
QSLinear.py:13-113, QConv.py:13-166, base/QFuncs/quant_basic.py:7-80).

* ``SLinear`` — Linear whose input keeps only values above the per-row k-th smallest
  magnitude (``sparse_ratio`` of the row zeroed).
* ``QSLinear`` — fake-quantised Linear (input and weight quantise→dequantise with the
  assigned formats, gradient of the output quantised with the input format) plus the same
  input sparsification.
* ``QConv2d`` — conv2d with fake-quantised input and weight (format along the channel
  dim) and the output gradient quantised with the input format.
* ``quant_block_float`` — block floating point with a shared exponent per group of
  ``blk_size`` values (and per outer block of ``blk_outer_size`` groups), either
  integer mantissas (``exp_bits == 0``) or small floats with private exponents.

None of these is on an OSP-Next model path (the model uses HiF8 linears, quant/hif8.py);
they complete the library API for code that builds on it.
"""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional, Union

import torch
import torch.nn as nn
import torch.nn.functional as F

from .hif8 import QType, quant_dequant_float


# ---------------------------------------------------------------------------- block float

@dataclass(frozen=True)
class BlockFloatFormat:
    """Fields of a block-floating-point format (names as in the library's QType)."""
    exp_bits: int                 # 0: integer mantissas under the shared exponent
    man_bits: int
    k_bits: int                   # range of a group's exponent below its block's largest
    blk_size: int = 1             # values per group (one shared exponent)
    blk_outer_size: int = 1       # groups per outer block
    exp_max: int = 0
    exp_min: int = 0
    k_max: int = 127
    fp_val_max: float = float("inf")
    man_shift_bit: int = 0
    exp_offset: int = 0
    do_carry: bool = True


def quant_block_float(x: torch.Tensor, fmt: BlockFloatFormat, qdim: int = -1) -> torch.Tensor:
    """Quantise→dequantise ``x`` along ``qdim`` (whose size must be a multiple of
    blk_size·blk_outer_size) to the block float ``fmt``."""
    qdim = qdim if qdim < 0 else qdim - x.dim()
    x = x.unflatten(qdim, (-1, fmt.blk_outer_size, fmt.blk_size))
    mag, sgn = x.abs(), torch.sign(x)
    lo, hi = -fmt.k_max - fmt.exp_offset, fmt.k_max - fmt.exp_offset
    top = mag.amax(dim=qdim, keepdim=True)                          # largest value of each group
    if fmt.exp_bits == 0:
        e_grp = (torch.floor(torch.log2(top + 9.6e-7)) - fmt.exp_max).clip(lo, hi)
        if fmt.do_carry:                                            # a mantissa rounding up to 2^m carries
            carry = (torch.floor(mag / torch.exp2(e_grp) + 0.5) - (2 ** fmt.man_bits - 1)).clip(0, 1)
            e_grp = e_grp + carry.amax(dim=qdim, keepdim=True)
    else:
        lg = torch.log2(top + 9.6e-7)
        e_grp = ((torch.floor(lg + 0.5) if fmt.do_carry else torch.floor(lg)) - fmt.exp_max).clip(lo, hi)
    # groups of a block stay within 2^k_bits − 1 exponents of the block's largest
    e = e_grp.clip(e_grp.amax(dim=qdim - 1, keepdim=True) - (2 ** fmt.k_bits - 1)).clip(lo, hi)
    if fmt.exp_bits == 0:
        mant = torch.floor(mag / torch.exp2(e) + 0.5).clip(0, 2 ** fmt.man_bits - 1)
        out = sgn * mant * torch.exp2(e)
        out = torch.where(mag < (2 - 2 ** (-fmt.man_bits)) * 2 ** (lo + 1), torch.zeros_like(out), out)
        limit = 2 ** (hi + fmt.exp_max) * (2 - 2 ** -fmt.man_bits)
        bad = (torch.isnan(mag) | torch.isinf(mag)).any(dim=qdim, keepdim=True)
        bad = bad | (mag >= limit).any(dim=qdim, keepdim=True).any(dim=qdim - 1, keepdim=True)
        out = torch.where(bad.expand_as(out), torch.full_like(out, float("nan")), out)
    else:
        xb = mag / torch.exp2(e)
        pe = torch.floor(torch.log2(xb + 9.6e-7)).clip(fmt.exp_min, fmt.exp_max)
        scale = 2.0 ** fmt.man_shift_bit
        v = (torch.floor(xb / torch.exp2(pe) * scale + 0.5) / scale * torch.exp2(pe)).clip(-fmt.fp_val_max,
                                                                                         fmt.fp_val_max)
        v = torch.where((e < -127).expand_as(v), torch.zeros_like(v), v)
        out = sgn * torch.exp2(e) * v
    return out.flatten(qdim - 2, qdim)


def quant_py(x: torch.Tensor, fmt: BlockFloatFormat, qdim: int) -> torch.Tensor:
    """The library's name for :func:`quant_block_float`."""
    return quant_block_float(x, fmt, qdim)


# ---------------------------------------------------------------------------- layers

def _as_qtype(q: Union[QType, str]) -> QType:
    return QType(q) if isinstance(q, str) else q.copy()


def _qdq(x, q: Optional[QType]):
    return x if q is None else quant_dequant_float(x, q)


def sparsify_rows(x: torch.Tensor, ratio: float) -> torch.Tensor:
    """Zero every value whose magnitude is ≤ the k-th smallest of its row, k = ⌊ratio·C⌋."""
    if ratio <= 0:
        return x
    k = int(x.shape[-1] * ratio)
    if k <= 0:
        raise ValueError(f"sparse ratio {ratio} keeps every value of a row of {x.shape[-1]}")
    thr = torch.kthvalue(x.abs().float(), k=k, dim=-1).values.to(x.dtype)
    return x.masked_fill(x.abs() <= thr.unsqueeze(-1), 0.0)


class _LinearQS(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, q_w, q_in, ratio):
        x_q = sparsify_rows(_qdq(x, q_in), ratio)
        w_q = _qdq(w, q_w)
        ctx.save_for_backward(x_q, w_q)
        ctx.q_in, ctx.has_b = q_in, b is not None
        return F.linear(x_q, w_q, b)

    @staticmethod
    def backward(ctx, g):
        x_q, w_q = ctx.saved_tensors
        gq = _qdq(g, ctx.q_in)
        dx = gq @ w_q
        dw = gq.flatten(0, -2).t() @ x_q.flatten(0, -2)
        db = g.flatten(0, -2).sum(0) if ctx.has_b else None
        return dx, dw, db, None, None, None


class _QuantParamsMixin:
    def _init_q(self):
        self.qparams: Optional[QType] = None
        self.in_qparams: Optional[QType] = None
        self._quant_grad = True

    def set_quant_grad(self, value: bool):
        self._quant_grad = value

    def assign_qparams(self, q):
        self.qparams = _as_qtype(q).dim_(self._qdim)

    def assign_input_qparams(self, q):
        self.in_qparams = _as_qtype(q).dim_(self._qdim)

    def transfer(self, layer):
        with torch.no_grad():
            self.to(layer.weight.device, layer.weight.dtype)
            self.weight.copy_(layer.weight)
            if self.bias is not None and layer.bias is not None:
                self.bias.copy_(layer.bias)


class SLinear(nn.Linear):
    """Linear with row-wise input sparsification (``sparse_ratio`` of each row zeroed)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, sparse_ratio: float = 0.0):
        super().__init__(in_features, out_features, bias)
        self.sparse_ratio = sparse_ratio

    def forward(self, x):
        return F.linear(sparsify_rows(x, self.sparse_ratio), self.weight, self.bias)

    def transfer(self, layer: nn.Linear):
        _QuantParamsMixin.transfer(self, layer)


class QSLinear(nn.Linear, _QuantParamsMixin):
    """Fake-quantised + sparsified Linear: x and W quantise→dequantise in forward (input
    format defaults to the weight format), the output gradient with the input format."""
    _qdim = -1

    def __init__(self, in_features: int, out_features: int, bias: bool = True, sparse_ratio: float = 0.0):
        super().__init__(in_features, out_features, bias)
        self.sparse_ratio = sparse_ratio
        self._init_q()

    def forward(self, x):
        if self.qparams is None:
            raise RuntimeError("QSLinear: assign quant params (QType) first")
        q_in = self.in_qparams or self.qparams
        return _LinearQS.apply(x.contiguous(), self.weight, self.bias, self.qparams, q_in, self.sparse_ratio)


class _QuantFwd(torch.autograd.Function):
    """Quantise in forward, pass the gradient through."""

    @staticmethod
    def forward(ctx, x, q):
        return _qdq(x, q)

    @staticmethod
    def backward(ctx, g):
        return g, None


class _QuantBwd(torch.autograd.Function):
    """Identity in forward, quantise the gradient in backward."""

    @staticmethod
    def forward(ctx, x, q):
        ctx.q = q
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return _qdq(g, ctx.q), None


class QConv2d(nn.Conv2d, _QuantParamsMixin):
    """conv2d on fake-quantised input and weight (format along channels), the output
    gradient quantised with the input format; bias added after."""
    _qdim = 1

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias: bool = True):
        super().__init__(in_channels, out_channels, kernel_size, stride=stride, padding=padding,
                         dilation=dilation, groups=groups, bias=bias)
        self._init_q()

    def forward(self, x):
        if self.qparams is None:
            raise RuntimeError("QConv2d: assign quant params (QType) first")
        q_in = self.in_qparams or self.qparams
        xq = _QuantFwd.apply(x.contiguous(), q_in)
        wq = _QuantFwd.apply(self.weight, self.qparams)
        out = F.conv2d(xq, wq, None, self.stride, self.padding, self.dilation, self.groups)
        if self._quant_grad:
            out = _QuantBwd.apply(out, q_in)
        return out if self.bias is None else out + self.bias[:, None, None]
