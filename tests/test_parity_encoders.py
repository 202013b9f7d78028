"""Frozen encoders vs the reference with identical weights (CPU, fp32):
Wan VAE chunked encode / per-frame decode, umT5 encoder with a padding mask."""
import torch

from osp_next_b200.models import t5 as mt5
from osp_next_b200.models import vae as mvae


def test_vae_matches_reference(reference):
    import ospnext.modules.vae as rvae
    torch.manual_seed(0)
    cfg = dict(dim=8, z_dim=4, dim_mult=[1, 2, 4, 4], num_res_blocks=1, attn_scales=[],
               temperal_downsample=[False, True, True])
    a, b = rvae.WanVAE_(**cfg).eval(), mvae.WanVAE_(**cfg).eval()
    with torch.no_grad():
        for p in a.parameters():
            p.copy_(torch.randn_like(p) * 0.1)
    b.load_state_dict(a.state_dict(), strict=True)
    x = torch.randn(1, 3, 9, 32, 32)
    sc = [torch.randn(4), torch.rand(4) + 0.5]
    with torch.no_grad():
        za, zb = a.encode(x, sc), b.encode(x, sc)
        assert torch.allclose(za, zb, atol=1e-6)
        assert torch.allclose(a.decode(za, sc), b.decode(za, sc), atol=1e-6)


def test_t5_matches_reference(reference):
    import ospnext.modules.t5 as rt5
    torch.manual_seed(0)
    kw = dict(vocab=100, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, num_buckets=32,
              shared_pos=False, dropout=0.0)
    a, b = rt5.T5Encoder(**kw).eval(), mt5.T5Encoder(**kw).eval()
    b.load_state_dict(a.state_dict(), strict=True)
    ids = torch.randint(0, 100, (2, 20))
    m = torch.ones(2, 20, dtype=torch.long)
    m[1, 12:] = 0
    with torch.no_grad():
        assert torch.allclose(a(ids, m), b(ids, m), atol=1e-5)
