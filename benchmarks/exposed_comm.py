"""Exposed communication time of a training step (analysis tool, not a bench number).

``torchrun --nproc-per-node N -m benchmarks.exposed_comm [bench.py train flags]``
runs the same trainer as ``bench.py --mode train`` (``--impl reference``: the reference arm's
training step, ``baseline/ref_train.py``) and records, on every rank, the device kernels of
the timed steps with the PyTorch profiler.  Per step:

  busy     union of the intervals of all kernels
  compute  union of the intervals of kernels that are not communication (NCCL kernels,
           and the NVLink barrier / gather / reduce-scatter / pull kernels of the P2P
           collectives and the SSP exchange)
  exposed  busy − compute: time in which only communication runs on the device

The max over ranks is printed as one JSON line.  Timings come from a profiled run and are
only used to split a step into compute and exposed communication.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMM_MARKERS = ("nccl", "p2p_barrier", "p2p_gather", "p2p_reduce_scatter", "p2p_pull")


def _union(iv):
    iv = sorted(iv)
    tot, cur_s, cur_e = 0.0, None, None
    for s, e in iv:
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                tot += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    if cur_e is not None:
        tot += cur_e - cur_s
    return tot


def main():
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "train"))
    import bench
    import train_osp
    args = bench.parse()
    rank, world, local = bench.init_dist(args.gpus, "cpu:gloo,cuda:nccl")
    cfg = bench.train_config(args, world, tempfile.mkdtemp(prefix="osp_comm_"))
    total = args.warmup + args.steps
    prof = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA],
                                  schedule=torch.profiler.schedule(wait=0, warmup=args.warmup - 1, active=args.steps,
                                                                   repeat=1))
    prof.start()
    if args.impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        import ref_train
        ref_train.train(cfg, lambda it, ms, tok: prof.step())
    else:
        train_osp.main(cfg, on_step=lambda it, ms, tok: prof.step())
    prof.stop()
    kernels = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    comm = [(e.time_range.start, e.time_range.end) for e in kernels
            if any(m in e.name.lower() for m in COMM_MARKERS)]
    comp = [(e.time_range.start, e.time_range.end) for e in kernels
            if not any(m in e.name.lower() for m in COMM_MARKERS)]
    busy = _union(comm + comp) / 1000.0 / args.steps
    compute = _union(comp) / 1000.0 / args.steps
    t = torch.tensor([busy, compute, busy - compute, _union(comm) / 1000.0 / args.steps], device="cuda",
                     dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({"bench": "exposed_comm_per_train_step", "impl": args.impl, "model": args.model,
                          "n_gpus": world, "fsdp_comm": args.fsdp_comm if args.impl == "ours" else "nccl",
                          "steps_profiled": args.steps,
                          "ms_device_busy": round(t[0].item(), 2), "ms_compute": round(t[1].item(), 2),
                          "ms_exposed_comm": round(t[2].item(), 2), "ms_comm_kernels": round(t[3].item(), 2),
                          "note": "max over ranks; from a profiled run"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
