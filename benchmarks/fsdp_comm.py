"""Bandwidth of the NVLink pull all-gather / reduce-scatter used for FSDP, against NCCL.

``torchrun --nproc-per-node N -m benchmarks.fsdp_comm``: one 14B block's
worth of data (351 M parameters: 702 MB bf16 gathered, 1.40 GB fp32 reduce-scattered, and
the bf16-gradient reduce-scatter with fp32 accumulation that the bf16 blocks use: 702 MB
pulled, fp32 shard out), CUDA events on every rank, min of 5 after warm-up, max over ranks.
Roofline = bytes each rank pulls over NVLink ((N−1)/N of the buffer) ÷ 770 GB/s per
direction.  The NCCL column of the bf16 case is what FSDP does without the fused pull: cast
the bf16 gradients into an fp32 buffer, then an fp32 reduce-scatter.
"""
from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from osp_next_b200 import ops
from osp_next_b200.parallel.fsdp_comm import _Arena

NVLINK_GBS = 770.0
BLOCK_PARAMS = 351_000_000


def _time(fn, reps=5):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    best = 1e30
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b))
    t = torch.tensor([best], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    shard = (BLOCK_PARAMS + world - 1) // world
    shard = (shard + 63) // 64 * 64
    res = {"bench": "fsdp_collectives", "world": world, "params": shard * world}
    for name, dtype in (("all_gather", torch.bfloat16), ("reduce_scatter", torch.float32),
                        ("reduce_scatter_bf16", torch.bfloat16)):
        esz = torch.empty(0, dtype=dtype).element_size()
        arena = _Arena(dist.group.WORLD, shard * world * esz, 2, dev)
        buf = arena.slot(shard * world, dtype)
        buf.normal_()
        off = arena.offset(buf)
        ref_in = torch.randn(shard * world, device=dev).to(dtype)
        if name == "all_gather":
            def p2p():
                arena.barrier(off)
                ops.ext().p2p_gather(arena.bases, off, shard * esz, arena.rank, world, arena.abort_ptr)
            out_nccl = torch.empty(shard * world, dtype=dtype, device=dev)

            def nccl():
                dist.all_gather_into_tensor(out_nccl, ref_in[rank * shard:(rank + 1) * shard])
        elif name == "reduce_scatter_bf16":
            out = torch.empty(shard, dtype=torch.float32, device=dev)

            def p2p():
                arena.barrier(off)
                ops.ext().p2p_reduce_scatter_bf16(out, arena.bases, off, shard, arena.rank, world, 1.0 / world,
                                                  arena.abort_ptr)
            out_nccl = torch.empty(shard, dtype=torch.float32, device=dev)
            staged = torch.empty(shard * world, dtype=torch.float32, device=dev)

            def nccl():
                staged.copy_(ref_in)
                dist.reduce_scatter_tensor(out_nccl, staged, op=dist.ReduceOp.AVG)
        else:
            out = torch.empty(shard, dtype=dtype, device=dev)

            def p2p():
                arena.barrier(off)
                ops.ext().p2p_reduce_scatter_f32(out, arena.bases, off, shard, arena.rank, world, 1.0 / world,
                                                 arena.abort_ptr)
            out_nccl = torch.empty(shard, dtype=dtype, device=dev)

            def nccl():
                dist.reduce_scatter_tensor(out_nccl, ref_in, op=dist.ReduceOp.AVG)
        t_p2p, t_nccl = _time(p2p), _time(nccl)
        pulled = (world - 1) * shard * esz
        roof = pulled / (NVLINK_GBS * 1e6)
        res[name] = {"mb": round(shard * world * esz / 1e6, 1), "ms_p2p": round(t_p2p, 3),
                     "ms_nccl": round(t_nccl, 3), "roofline_ms": round(roof, 3),
                     "frac_of_roofline_p2p": round(roof / t_p2p, 3), "frac_of_roofline_nccl": round(roof / t_nccl, 3)}
        dist.barrier()
        arena.close()
    res["device_error"] = ops.ext().get_error(local, True)
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
