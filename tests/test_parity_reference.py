"""Module parity: our DiT vs the reference's OSPNextModel with the same weights (CPU, fp32).

The reference's attention casts q/k/v to bf16 even on CPU (attention.py:460-478),
so outputs agree to bf16-level tolerance.
"""
import pytest
import torch

from osp_next_b200.models.osp_next import OSPNextModel


def _pair(reference, **cfg):
    osp, _ = reference
    torch.manual_seed(0)
    theirs = osp.OSPNextModel(**cfg).eval()
    ours = OSPNextModel(**cfg).eval()
    missing, unexpected = ours.load_state_dict(theirs.state_dict(), strict=True), None
    return theirs, ours


@pytest.mark.parametrize("cfg,shape", [
    (dict(dim=256, ffn_dim=1024, num_heads=4, num_layers=2, text_len=32, skiparse_model_type="dual_end",
          sparse_ratio=2, num_full_blocks=0), (1, 16, 5, 32, 32)),
    (dict(dim=128, ffn_dim=256, num_heads=2, num_layers=8, text_len=16, skiparse_model_type="dual_end",
          sparse_ratio=2, num_full_blocks=4), (2, 16, 3, 18, 22)),      # padded grid: 9x11 patches
    (dict(dim=128, ffn_dim=256, num_heads=2, num_layers=4, text_len=16, skiparse_model_type="full"),
     (1, 16, 2, 8, 12)),
])
def test_forward_matches_reference(reference, cfg, shape):
    theirs, ours = _pair(reference, **cfg)
    torch.manual_seed(1)
    x = torch.randn(*shape)
    t = torch.rand(shape[0]) * 1000
    ctx = torch.randn(shape[0], cfg["text_len"], 4096)
    with torch.no_grad():
        a = theirs(x, t, ctx)
        b = ours(x, t, ctx)
    assert a.shape == b.shape
    err = (a - b).abs().max().item()
    scale = a.abs().max().item()
    assert err <= 2e-2 * scale + 1e-3, (err, scale)


def test_state_dict_keys_match(reference):
    osp, _ = reference
    cfg = dict(dim=128, ffn_dim=256, num_heads=2, num_layers=8, text_len=16, skiparse_model_type="dual_end",
               sparse_ratio=2, num_full_blocks=4)
    a = osp.OSPNextModel(**cfg).state_dict()
    b = OSPNextModel(**cfg).state_dict()
    assert list(a.keys()) == list(b.keys())
    for k in a:
        assert a[k].shape == b[k].shape, k


def test_backward_matches_reference(reference):
    cfg = dict(dim=128, ffn_dim=256, num_heads=2, num_layers=2, text_len=16, skiparse_model_type="dual_end",
               sparse_ratio=2, num_full_blocks=0)
    theirs, ours = _pair(reference, **cfg)
    theirs.train(); ours.train()
    torch.manual_seed(2)
    x = torch.randn(1, 16, 2, 16, 16)
    t = torch.tensor([300.0])
    ctx = torch.randn(1, 16, 4096)
    theirs(x, t, ctx).pow(2).mean().backward()
    ours(x, t, ctx).pow(2).mean().backward()
    ga = dict(theirs.named_parameters())
    for n, p in ours.named_parameters():
        g1, g2 = ga[n].grad, p.grad
        assert g2 is not None, n
        rel = (g1 - g2).norm() / (g1.norm() + 1e-12)
        assert rel < 5e-2, (n, rel.item())
