"""Multi-GPU sequence parallelism on NCCL vs one GPU (skipped with fewer than 2 GPUs).

Ranks are separate processes, one per GPU; NVLS is disabled (NCCL_NVLS_ENABLE=0) and a
short process-group timeout bounds every collective.
"""
import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(dim=256, ffn_dim=512, num_heads=4, num_layers=8, text_len=16, skiparse_model_type="dual_end",
           sparse_ratio=2, num_full_blocks=4)
SHAPE = (1, 16, 3, 24, 32)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _build(device):
    from osp_next_b200.models.osp_next import OSPNextModel
    torch.manual_seed(0)
    with torch.device(device):
        m = OSPNextModel(**CFG)
    return m.to(torch.bfloat16).eval()


def _inputs(device):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(*SHAPE, generator=g).to(device, torch.bfloat16)
    t = torch.tensor([500.0], device=device)
    ctx = torch.randn(1, CFG["text_len"], 4096, generator=g).to(device, torch.bfloat16)
    return x, t, ctx


def _worker(rank, world, port, ssp, exchange, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from osp_next_b200.parallel.sp import attach_sp, build_sp_groups
    dev = torch.device("cuda", rank)
    m = _build(dev)
    attach_sp(m, build_sp_groups(CFG["num_heads"], skiparse_sp_size=ssp, sp_size=1))
    if exchange == "p2p":
        from osp_next_b200.parallel.sp import enable_p2p_exchange
        enable_p2p_exchange(m, SHAPE[0], (SHAPE[2], SHAPE[3] // 2, SHAPE[4] // 2), dev)
    x, t, ctx = _inputs(dev)
    with torch.no_grad():
        y = m(x, t, ctx)
    from osp_next_b200 import ops
    torch.save({"y": y.float().cpu(), "err": ops.ext().get_error(rank, True)}, os.path.join(out_dir, f"r{rank}.pt"))
    if m.parallel is not None and m.parallel.p2p is not None:
        m.parallel.p2p.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
@pytest.mark.parametrize("ssp", [2, 4])
def test_ssp_matches_single_gpu(ssp, exchange):
    if torch.cuda.device_count() < ssp:
        pytest.skip(f"needs {ssp} GPUs")
    m = _build("cuda:0")
    x, t, ctx = _inputs("cuda:0")
    with torch.no_grad():
        y1 = m(x, t, ctx).float().cpu()
    del m
    torch.cuda.empty_cache()
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(ssp, _port(), ssp, exchange, d), nprocs=ssp, join=True,
                           start_method="spawn")
        for r in range(ssp):
            o = torch.load(os.path.join(d, f"r{r}.pt"))
            assert o["err"] == 0
            rel = (o["y"] - y1).norm() / y1.norm()
            assert rel < 2e-2, (r, rel)


def _train_model(device, heads):
    from osp_next_b200.models.osp_next import OSPNextModel
    torch.manual_seed(0)
    with torch.device(device):
        m = OSPNextModel(**dict(CFG, num_heads=heads))
        m.head.head.weight.data.normal_(std=0.02)
    return m.train()


def _train_inputs(device):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(*SHAPE, generator=g).to(device)
    ctx = torch.randn(1, CFG["text_len"], 4096, generator=g).to(device)
    tgt = torch.randn(*SHAPE, generator=g).to(device)
    return x, torch.tensor([400.0], device=device), ctx, tgt


def _train_step(m, dev):
    x, t, ctx, tgt = _train_inputs(dev)
    loss = (m(x, t, ctx).float() - tgt).pow(2).mean()
    loss.backward()
    return loss.detach(), {n: p.grad.float().cpu() for n, p in m.named_parameters() if p.grad is not None}


def _train_sp_worker(rank, world, port, ssp, ul, heads, exchange, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from osp_next_b200 import ops
    from osp_next_b200.parallel.sp import attach_sp, build_sp_groups, enable_p2p_exchange
    m = _train_model(dev, heads)
    attach_sp(m, build_sp_groups(heads, skiparse_sp_size=ssp, sp_size=ul))
    if exchange == "p2p":
        enable_p2p_exchange(m, SHAPE[0], (SHAPE[2], SHAPE[3] // 2, SHAPE[4] // 2), dev, limit_s=30.0)
    loss, grads = _train_step(m, dev)
    torch.save({"loss": loss.item(), "grads": grads, "err": ops.ext().get_error(rank, True)},
               os.path.join(out_dir, f"t{rank}.pt"))
    if m.parallel is not None and m.parallel.p2p is not None:
        m.parallel.p2p.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("ssp,ul,heads", [(2, 1, 4), (2, 2, 4), (4, 1, 2)])
def test_training_sp_exchange_matches_single_gpu(ssp, ul, heads):
    """One training step (forward + backward) under SSP, Ulysses × SSP and SSP with
    replicated dense rows (full_sp < world), with the layout changes and head all-to-alls
    over NVLink peer memory and over NCCL: the loss matches one GPU and the ranks'
    gradients sum to world × the one-GPU gradient (the all-gather's SUM backward); the
    two transports agree with each other more tightly."""
    world = ssp * ul
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    m = _train_model("cuda:0", heads)
    loss1, g1 = _train_step(m, torch.device("cuda:0"))
    del m
    torch.cuda.empty_cache()
    res = {}
    for exchange in ("nccl", "p2p"):
        with tempfile.TemporaryDirectory() as d:
            mp.start_processes(_train_sp_worker, args=(world, _port(), ssp, ul, heads, exchange, d), nprocs=world,
                               join=True, start_method="spawn")
            res[exchange] = [torch.load(os.path.join(d, f"t{r}.pt")) for r in range(world)]
    for exchange, outs in res.items():
        for o in outs:
            assert o["err"] == 0
            assert abs(o["loss"] - loss1.item()) <= 1e-2 * abs(loss1.item()), (exchange, o["loss"], loss1.item())
        for n, g in g1.items():
            s = sum(o["grads"][n] for o in outs) / world
            rel = ((s - g).norm() / g.norm().clamp_min(1e-12)).item()
            assert rel < 5e-2, (exchange, n, rel)
    for n in g1:
        a = sum(o["grads"][n] for o in res["p2p"])
        b = sum(o["grads"][n] for o in res["nccl"])
        rel = ((a - b).norm() / b.norm().clamp_min(1e-12)).item()
        assert rel < 1e-2, (n, rel)


def _fsdp_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from torch.distributed.device_mesh import init_device_mesh
    from osp_next_b200.models.osp_next import OSPNextAttentionBlock, OSPNextModel, WanLayerNorm, WanRMSNorm
    from osp_next_b200.parallel.fsdp import FSDP2_mix_wrapper
    from osp_next_b200.parallel.fsdp_comm import check, close, enable_p2p_fsdp
    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("fsdp",))
    out = {}
    for mode in ("nccl", "p2p"):
        torch.manual_seed(0)
        with torch.device(dev):
            m = OSPNextModel(dim=256, ffn_dim=512, num_heads=2, num_layers=4, text_len=16,
                             skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=0)
            m.head.head.weight.data.normal_(std=0.02)
        FSDP2_mix_wrapper(m, mesh, torch.bfloat16, main_block_to_half=OSPNextAttentionBlock,
                          blocks_to_float=[WanLayerNorm, WanRMSNorm])
        arenas = enable_p2p_fsdp(list(m.blocks), mesh.get_group(), device=dev) if mode == "p2p" else None
        opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
        g = torch.Generator().manual_seed(10 + rank)
        losses = []
        # no host synchronisation between steps: slot reuse in the NVLink arenas is ordered
        # on the GPU alone
        for _ in range(8):
            x = torch.randn(1, 16, 3, 16, 16, generator=g).to(dev, non_blocking=True)
            ctx = torch.randn(1, 16, 4096, generator=g).to(dev, non_blocking=True)
            loss = m(x, torch.tensor([400.0], device=dev), ctx).float().pow(2).mean()
            loss.backward()
            opt.step()
            opt.zero_grad()
            losses.append(loss.detach())
        losses = [v.item() for v in losses]
        if arenas is not None:
            check(arenas, rank)
            dist.barrier()
            close(arenas)
        out[mode] = (losses, sum(p.to_local().float().sum().item() for p in m.parameters()))
        if arenas is not None:
            out["rs_grad_bytes"] = arenas[1].grad_bytes     # bf16 blocks: bf16 reduce-scatter input
    torch.save(out, os.path.join(out_dir, f"f{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fsdp_p2p_collectives_match_nccl():
    """FSDP2 training steps with the NVLink pull all-gather / reduce-scatter give the same
    losses and parameters as with NCCL collectives."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_fsdp_worker, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            o = torch.load(os.path.join(d, f"f{r}.pt"))
            (ln, pn), (lp, pp) = o["nccl"], o["p2p"]
            assert o["rs_grad_bytes"] == 2
            for a, b in zip(ln, lp):
                assert abs(a - b) <= 1e-4 * max(1.0, abs(a)), (ln, lp)
            assert abs(pn - pp) <= 1e-3 * max(1.0, abs(pn)), (pn, pp)


def _rs_bf16_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from osp_next_b200 import ops
    from osp_next_b200.parallel.fsdp_comm import _Arena
    res = {}
    for shard in (4096, 1000, 77):                 # vector path, scalar path (shard % 8 != 0)
        arena = _Arena(dist.group.WORLD, shard * world * 2, 2, dev)
        buf = arena.slot(shard * world, torch.bfloat16)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        buf.copy_(torch.randn(shard * world, device=dev, generator=g).to(torch.bfloat16))
        ref_in = buf.float().clone()
        out = torch.empty(shard, dtype=torch.float32, device=dev)
        arena.barrier(arena.offset(buf))
        ops.ext().p2p_reduce_scatter_bf16(out, arena.bases, arena.offset(buf), shard, rank, world, 1.0 / world,
                                          arena.abort_ptr)
        ref = torch.empty(shard, dtype=torch.float32, device=dev)
        dist.reduce_scatter_tensor(ref, ref_in, op=dist.ReduceOp.AVG)
        torch.cuda.synchronize()
        res[shard] = (out - ref).abs().max().item()
        del buf
        dist.barrier()
        arena.close()
    res["err"] = ops.ext().get_error(rank, True)
    torch.save(res, os.path.join(out_dir, f"rs{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_reduce_scatter_bf16_matches_nccl_fp32():
    """The bf16-gradient pull reduce-scatter (fp32 accumulation) equals NCCL's fp32
    reduce-scatter of the same values cast to fp32, up to summation order."""
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rs_bf16_worker, args=(2, _port(), d), nprocs=2, join=True, start_method="spawn")
        for r in range(2):
            o = torch.load(os.path.join(d, f"rs{r}.pt"))
            assert o["err"] == 0
            for shard in (4096, 1000, 77):
                assert o[shard] <= 1e-6, o
