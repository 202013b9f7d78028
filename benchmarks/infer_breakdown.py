"""Where a sampling step's time goes at N GPUs (analysis tool, not a bench number).

``torchrun --nproc-per-node N -m benchmarks.infer_breakdown [bench.py flags]`` builds the
same model, layout (1: batch-2 CFG; 2: CFG-parallel; 4: CFG-2 × SSP-2; 8: CFG-2 × SSP-4)
and sampler as ``bench.py`` and records the device kernels of ``--steps`` denoising steps
with the PyTorch profiler.  Kernels are grouped by name into categories:

  gemm        tcgen05 GEMMs (projections, FFN, embeddings, head)
  attention   attention forward kernels
  rows        LN-modulate, RMSNorm, q/k-norm + RoPE, CFG + Euler, other elementwise
  p2p         NVLink exchange barrier (the exchange stores run inside the FFN-down GEMM)
  nccl        NCCL kernels: dense-block Ulysses all-to-all, boundary redistribution /
              gather, CFG velocity swap
  other       everything else (PyTorch copies / indexing)

Per step it reports each category's summed kernel time, the device-busy time (union of
all kernel intervals), and the exposed communication: busy time during which only p2p /
NCCL kernels run.  Max over ranks, one JSON line.  Timings come from a profiled run and are
only used to split a step, never as the bench value.
"""
from __future__ import annotations

import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CATS = (("nccl", ("nccl",)), ("p2p", ("p2p_barrier",)), ("attention", ("attn_fwd",)),
        ("gemm", ("gemm_kernel",)),
        ("rows", ("ln_modulate", "rms_norm", "qk_norm_rope", "cfg_euler", "layer_norm", "gated_add")))


def category(name: str) -> str:
    n = name.lower()
    for cat, keys in CATS:
        if any(k in n for k in keys):
            return cat
    return "other"


def _union(iv):
    iv = sorted(iv)
    tot, s0, e0 = 0.0, None, None
    for s, e in iv:
        if e0 is None or s > e0:
            if e0 is not None:
                tot += e0 - s0
            s0, e0 = s, e
        else:
            e0 = max(e0, e)
    return tot + (e0 - s0 if e0 is not None else 0.0)


def main():
    sys.path.insert(0, ROOT)
    import bench
    args = bench.parse()
    rank, world, local = bench.init_dist(args.gpus, "nccl")
    args.no_e2e = True
    captured = {}

    def run(fn_steps):
        prof = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA])
        with prof:
            fn_steps()
            torch.cuda.synchronize()
        captured["events"] = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]

    bench.run_ours(args, rank, world, local, profile_hook=run)
    ev = captured["events"]
    per = {c: 0.0 for c, _ in CATS}
    per["other"] = 0.0
    by_name = {}
    comm_iv, comp_iv = [], []
    for e in ev:
        c = category(e.name)
        d = (e.time_range.end - e.time_range.start)
        per[c] += d
        by_name[e.name] = by_name.get(e.name, 0.0) + d
        (comm_iv if c in ("nccl", "p2p") else comp_iv).append((e.time_range.start, e.time_range.end))
    steps = max(1, args.steps)
    busy = _union(comm_iv + comp_iv)
    exposed = busy - _union(comp_iv)
    vals = [per[c] for c in sorted(per)] + [busy, exposed]
    t = torch.tensor(vals, dtype=torch.float64, device="cuda") / 1000.0 / steps
    dist.all_reduce(t, op=dist.ReduceOp.MAX) if dist.is_initialized() else None
    if rank == 0:
        names = sorted(per)
        rec = {"bench": "inference_step_breakdown", "model": args.model, "n_gpus": world,
               "layout": {1: "single", 2: "cfg2", 4: "cfg2_ssp2", 8: "cfg2_ssp4"}[world],
               "exchange": args.exchange, "steps_profiled": steps,
               "ms_per_step_by_category": {n: round(t[i].item(), 2) for i, n in enumerate(names)},
               "ms_device_busy": round(t[len(names)].item(), 2),
               "ms_exposed_comm": round(t[len(names) + 1].item(), 2),
               "top_kernels_ms_per_step_rank0": [[k[:120], round(v / 1000.0 / steps, 3)] for k, v in
                                                 sorted(by_name.items(), key=lambda kv: -kv[1])[:25]],
               "note": "max over ranks; from a profiled run"}
        print(json.dumps(rec), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
