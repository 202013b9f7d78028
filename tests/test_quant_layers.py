"""Block-float quantiser vs the reference's quant_py (same format fields), and the sparse /
quantised Linear and Conv layers vs their definitions (CPU)."""
import importlib.util
import os

import pytest
import torch

from osp_next_b200.quant import layers as L
from osp_next_b200.quant.hif8 import QType, quant_dequant_float

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ref_quant_py():
    base = os.path.join(ROOT, "baseline", "_ref", "ospnext", "quant_cy_npu", "base")
    if not os.path.isdir(base):
        pytest.skip("reference not installed in baseline/_ref")
    import sys
    import types
    pkg = types.ModuleType("refq")
    pkg.__path__ = [base]
    sys.modules["refq"] = pkg
    spec = importlib.util.spec_from_file_location("refq.QType", os.path.join(base, "QType.py"))
    qt = importlib.util.module_from_spec(spec)
    sys.modules["refq.QType"] = qt
    spec.loader.exec_module(qt)
    fpkg = types.ModuleType("refq.QFuncs")
    fpkg.__path__ = [os.path.join(base, "QFuncs")]
    sys.modules["refq.QFuncs"] = fpkg
    spec = importlib.util.spec_from_file_location("refq.QFuncs.quant_basic", os.path.join(base, "QFuncs", "quant_basic.py"))
    qb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(qb)
    return qt.QType, qb.quant_py


FORMATS = [
    dict(exp_bits=0, man_bits=7, k_bits=2, blk_size=16, blk_outer_size=2, exp_max=6, exp_min=0, k_max=127),
    dict(exp_bits=0, man_bits=3, k_bits=1, blk_size=8, blk_outer_size=4, exp_max=2, exp_min=0, k_max=20,
         do_carry=False),
    dict(exp_bits=2, man_bits=1, k_bits=8, blk_size=32, blk_outer_size=1, exp_max=2, exp_min=0, k_max=127,
         fp_val_max=6.0, man_shift_bit=1),
    dict(exp_bits=3, man_bits=2, k_bits=3, blk_size=16, blk_outer_size=2, exp_max=4, exp_min=-2, k_max=60,
         fp_val_max=28.0, man_shift_bit=2, do_carry=False),
]


@pytest.mark.parametrize("f", FORMATS)
def test_block_float_matches_reference(f):
    RQ, quant_py = _ref_quant_py()
    q = RQ("custom")
    for k, v in f.items():
        setattr(q, k, v)
    fmt = L.BlockFloatFormat(**f)
    g = torch.Generator().manual_seed(0)
    for shape, dim in (((4, 64), -1), ((3, 128, 5), -2), ((2, 256), -1)):
        x = torch.randn(*shape, generator=g) * torch.exp2(torch.randint(-6, 6, shape, generator=g).float())
        a = L.quant_block_float(x, fmt, dim)
        b = quant_py(x.clone(), q, dim)
        assert torch.allclose(a, b, equal_nan=True), (a - b).abs().nan_to_num().max()


def test_sparse_and_quantised_layers():
    torch.manual_seed(0)
    x = torch.randn(3, 7, 32)
    s = L.SLinear(32, 16, sparse_ratio=0.25)
    y = s(x.clone())
    thr = torch.kthvalue(x.abs(), 8, dim=-1).values
    xs = torch.where(x.abs() <= thr[..., None], torch.zeros_like(x), x)
    assert torch.allclose(y, torch.nn.functional.linear(xs, s.weight, s.bias))
    q = L.QSLinear(32, 16)
    q.transfer(s)
    q.assign_qparams("bf16")
    xr = x.clone().requires_grad_(True)
    out = q(xr)
    out.sum().backward()
    exp = torch.nn.functional.linear(quant_dequant_float(x, QType("bf16")), quant_dequant_float(q.weight, QType("bf16")),
                                     q.bias)
    assert torch.allclose(out, exp) and xr.grad is not None and q.weight.grad is not None
    c = L.QConv2d(4, 6, 3, padding=1)
    c.assign_qparams("bf16")
    xi = torch.randn(2, 4, 9, 9, requires_grad=True)
    oc = c(xi)
    ref = torch.nn.functional.conv2d(xi.to(torch.bfloat16).float(), c.weight.to(torch.bfloat16).float(), c.bias,
                                     padding=1)
    assert torch.allclose(oc, ref, atol=1e-5)
    oc.sum().backward()
    assert xi.grad.shape == xi.shape
