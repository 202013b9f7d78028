"""Where a training step's device time goes (analysis tool, not a bench number).

``[torchrun --nproc-per-node N] python -m benchmarks.train_breakdown --mode train [bench.py
flags]`` runs the public trainer exactly as ``bench.py --mode train`` does and records
the device kernels of the timed steps (after ``--warmup``) with the PyTorch profiler.
Kernels are grouped by name:

  gemm        tcgen05 GEMMs (forward, dX, dW)
  attention   attention forward and backward kernels
  rows        LN-modulate, RMSNorm, q/k-norm + RoPE, gated add, GELU backward
  hif8        HiF8 amax / quantise-dequantise
  optimizer   fused AdamW, EMA, clipping norms
  p2p         NVLink exchange barrier / pulls and FSDP arena collectives
  nccl        NCCL kernels
  other       everything else (PyTorch elementwise, copies, reductions)

It prints one JSON line per rank 0: milliseconds per step per category (max over ranks)
and the 20 most expensive kernels on rank 0.  Timings come from a profiled run and only
split a step; the bench value is ``bench.py``'s.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CATS = (("nccl", ("nccl",)), ("p2p", ("p2p_",)), ("hif8", ("hif8",)),
        ("attention", ("attn_",)), ("gemm", ("gemm_kernel", "gemm_t")),
        ("optimizer", ("adamw", "ema", "multi_tensor", "foreach", "norm_sq")),
        ("rows", ("ln_modulate", "rms_norm", "qk_norm_rope", "gated_add", "gelu", "layer_norm")))


def category(name: str) -> str:
    n = name.lower()
    for cat, keys in CATS:
        if any(k in n for k in keys):
            return cat
    return "other"


def main():
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "train"))
    import bench
    args = bench.parse()
    rank, world, local = bench.init_dist(args.gpus, "nccl")
    cfg = bench.train_config(args, world, tempfile.mkdtemp(prefix="osp_train_breakdown_"))
    prof = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA])

    def on_step(it, ms, tok):
        if it == args.warmup:
            torch.cuda.synchronize()
            prof.start()
        if it == args.warmup + args.steps:
            torch.cuda.synchronize()
            prof.stop()

    import train_osp
    train_osp.main(cfg, on_step=on_step)
    per = {c: 0.0 for c, _ in CATS}
    per["other"] = 0.0
    by_name = {}
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        d = (e.time_range.end - e.time_range.start) / 1000.0
        per[category(e.name)] += d
        by_name[e.name] = by_name.get(e.name, 0.0) + d
    names = sorted(per)
    t = torch.tensor([per[n] for n in names], dtype=torch.float64, device="cuda") / max(1, args.steps)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        top = sorted(by_name.items(), key=lambda kv: -kv[1])[:20]
        print(json.dumps({"bench": "train_step_breakdown", "model": args.model, "quant": args.quant,
                          "n_gpus": world, "steps_profiled": args.steps,
                          "ms_per_step_by_category": {n: round(t[i].item(), 2) for i, n in enumerate(names)},
                          "ms_per_step_total": round(float(t.sum().item()), 2),
                          "top_kernels_ms_per_step": [(n[:120], round(v / max(1, args.steps), 3)) for n, v in top],
                          "note": "max over ranks per category; from a profiled run"}), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
