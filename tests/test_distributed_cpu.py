"""Sequence-parallel plumbing on CPU Gloo ranks vs a single process.

SSP (2, 4), Ulysses (2), SSP × Ulysses (2 × 2), dense blocks with full-blocks
Ulysses, padded grids; forward equality and the reference's gradient semantics
(every SP rank back-propagates the loss on the full output, so per-rank weight
gradients sum to ``sp_size ×`` the single-process gradient).
"""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CFGS = {
    "tiny": dict(dim=128, ffn_dim=256, num_heads=4, num_layers=2, text_len=16, skiparse_model_type="dual_end",
                 sparse_ratio=2, num_full_blocks=0),
    "dense8": dict(dim=128, ffn_dim=256, num_heads=4, num_layers=8, text_len=16, skiparse_model_type="dual_end",
                   sparse_ratio=2, num_full_blocks=4),
}


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfg_name, ssp, ul, shape, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from osp_next_b200.models.osp_next import OSPNextModel
    from osp_next_b200.parallel.sp import attach_sp, build_sp_groups
    torch.manual_seed(0)
    model = OSPNextModel(**CFGS[cfg_name])
    rt = build_sp_groups(CFGS[cfg_name]["num_heads"], skiparse_sp_size=ssp, sp_size=ul)
    attach_sp(model, rt)
    torch.manual_seed(1)
    x = torch.randn(*shape)
    t = torch.tensor([321.0] * shape[0])
    ctx = torch.randn(shape[0], CFGS[cfg_name]["text_len"], 4096)
    y = model(x, t, ctx)
    y.pow(2).mean().backward()
    grads = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    torch.save({"y": y.detach(), "grads": grads}, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _single(cfg_name, shape):
    from osp_next_b200.models.osp_next import OSPNextModel
    torch.manual_seed(0)
    model = OSPNextModel(**CFGS[cfg_name])
    torch.manual_seed(1)
    x = torch.randn(*shape)
    t = torch.tensor([321.0] * shape[0])
    ctx = torch.randn(shape[0], CFGS[cfg_name]["text_len"], 4096)
    y = model(x, t, ctx)
    y.pow(2).mean().backward()
    return y.detach(), {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}


@pytest.mark.parametrize("cfg_name,ssp,ul,shape", [
    ("tiny", 2, 1, (1, 16, 3, 16, 16)),
    ("tiny", 4, 1, (1, 16, 2, 18, 22)),        # padded grid
    ("tiny", 1, 2, (1, 16, 2, 16, 16)),
    ("tiny", 2, 2, (1, 16, 2, 16, 16)),
    ("dense8", 2, 1, (2, 16, 2, 16, 16)),
])
def test_sp_matches_single_process(cfg_name, ssp, ul, shape):
    world = ssp * ul
    y1, g1 = _single(cfg_name, shape)
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _port(), cfg_name, ssp, ul, shape, d), nprocs=world,
                           join=True, start_method="spawn")
        outs = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    for o in outs:
        assert torch.allclose(o["y"], y1, atol=2e-5, rtol=1e-4), (o["y"] - y1).abs().max()
    for n, g in g1.items():
        s = sum(o["grads"][n] for o in outs)
        assert torch.allclose(s, world * g, atol=1e-4, rtol=1e-3), (n, (s - world * g).abs().max())


def _t5_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from osp_next_b200.models import t5 as mt5
    torch.manual_seed(0)
    enc = mt5.T5Encoder(vocab=100, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, num_buckets=32,
                        shared_pos=False, dropout=0.0).eval()
    ref = {k: v.clone() for k, v in enc.state_dict().items()}
    model = mt5.T5EncoderModel(text_len=20, dtype=torch.float32, device="cpu", encoder=enc, use_fsdp=True,
                               device_mesh=mt5.t5_mesh(world, 8, "cpu"))
    assert any(hasattr(p, "to_local") for p in model.model.parameters())      # sharded
    ids = torch.randint(0, 100, (2, 20), generator=torch.Generator().manual_seed(3))
    m = torch.ones(2, 20, dtype=torch.long)
    m[1, 12:] = 0
    y = model(ids, m)
    torch.save({"y": y, "ref": ref, "ids": ids, "m": m}, os.path.join(out_dir, f"t5_{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_t5_fsdp_sharded_encoder_matches_unsharded():
    from osp_next_b200.models import t5 as mt5
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_t5_worker, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        outs = [torch.load(os.path.join(d, f"t5_{r}.pt")) for r in range(2)]
    enc = mt5.T5Encoder(vocab=100, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, num_buckets=32,
                        shared_pos=False, dropout=0.0).eval()
    enc.load_state_dict(outs[0]["ref"])
    single = mt5.T5EncoderModel(text_len=20, dtype=torch.float32, device="cpu", encoder=enc)
    exp = single(outs[0]["ids"], outs[0]["m"])
    for o in outs:
        assert torch.allclose(o["y"], exp, atol=1e-5), (o["y"] - exp).abs().max()
