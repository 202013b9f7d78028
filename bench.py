"""Headline benchmark: OSP-Next-14B T2V sampling, 81 frames 768×1280 (720P padded), 50 steps, CFG 5.

One *step* is one denoising step of the 50-step schedule: the conditional and the
unconditional 14B forward on 80 640 tokens plus the CFG + Euler update.  The
metric is seconds per video = (device time per step) × 50.  All steps of the
schedule cost the same, so timing K of them and multiplying by 50 is exact up to
noise; the timed steps are the first K of the real 50-step σ schedule.

Parallel layout per GPU count (strong scaling, one video):
  1: one GPU runs cond+uncond as one batch of 2
  2: CFG-parallel (cond on rank 0, uncond on rank 1; velocity swapped per step)
  4: CFG-parallel × Skiparse-SP 2;  8: CFG-parallel × Skiparse-SP 4
Dense blocks use Ulysses over the SSP ranks.

``--impl reference`` runs the unmodified reference (``baseline/_ref``) through its
own ``FlowMatchingScheduler.sample`` on the same shapes (see baseline/ref_harness.py).

``--mode train`` measures the other BASELINE metric instead: flow-matching training
tokens/s through ``train/train_osp.py`` (FSDP over all ranks, SSP up to 4, activation
checkpointing, adaptive clipping, fused AdamW, EMA), synthetic latents and text; the
reference arm runs the reference's own FSDP2 wrapper, model, scheduler, clipper, EMA and
``torch.optim.AdamW`` (baseline/ref_train.py).

Timing: W warm-up steps, then K steps between barrier + synchronize on every
rank; CUDA events on the launching stream; the max over ranks is reported.
Inputs are 1.6 GB of activations per step (> 126 MB L2), so L2 is not flushed.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_SEC_PER_VIDEO = None   # the reference publishes only speed-up ratios, no absolute sec/video
STEPS_PER_VIDEO = 50

PRESETS = {
    "14b": dict(dim=5120, ffn_dim=13824, freq_dim=256, in_dim=16, num_heads=40, num_layers=40, out_dim=16,
                text_len=512, skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=8),
    "1.3b": dict(dim=1536, ffn_dim=8960, freq_dim=256, in_dim=16, num_heads=12, num_layers=30, out_dim=16,
                 text_len=512, skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=8),
    "tiny": dict(dim=256, ffn_dim=1024, freq_dim=256, in_dim=16, num_heads=2, num_layers=2, out_dim=16,
                 text_len=32, skiparse_model_type="dual_end", sparse_ratio=2, num_full_blocks=0),
}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", choices=list(PRESETS), default="14b")
    p.add_argument("--frames", type=int, default=81)
    p.add_argument("--height", type=int, default=768)
    p.add_argument("--width", type=int, default=1280)
    p.add_argument("--guidance", type=float, default=5.0)
    p.add_argument("--shift", type=float, default=5.0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--mode", choices=["infer", "train"], default="infer",
                   help="infer: the sec/video headline; train: flow-matching training tokens/s")
    p.add_argument("--quant", choices=["none", "hif8"], default="none",
                   help="train mode: HiF8 fake-quant linears (BASELINE config 4) or plain bf16")
    p.add_argument("--loss-log", default=None, help="train mode: append per-step losses (JSONL) here")
    p.add_argument("--fsdp-comm", choices=["p2p", "nccl"], default="p2p",
                   help="train mode: FSDP block all-gather / reduce-scatter over NVLink peer memory or NCCL")
    p.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                   help="SSP layout exchange and Ulysses all-to-all: NVLink peer memory (fused GEMM-epilogue stores at inference, staged pulls otherwise) or NCCL")
    return p.parse_args()


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clocks / throttle reasons with nvidia-smi while the timed region runs."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return

        def rd():
            for line in self.proc.stdout:
                self.rows.append([c.strip() for c in line.split(",")])
        self.thread = threading.Thread(target=rd, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx.append(float(r[1]))
                for n, v in zip(names, r[3:7]):
                    if v.lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- helpers

def init_dist(n, backend="nccl"):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch with torchrun --nproc-per-node {n}")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(v: float) -> float:
    if not dist.is_initialized():
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier_sync():
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def latent_shape(args):
    return (1, 16, (args.frames - 1) // 4 + 1, args.height // 8, args.width // 8)


def tokens(args):
    _, _, T, H, W = latent_shape(args)
    return T * (H // 2) * (W // 2)


def layout_for(world: int):
    """(cfg, ssp) per GPU count."""
    return {1: (1, 1), 2: (2, 1), 4: (2, 2), 8: (2, 4)}[world]


# ----------------------------------------------------------------------------- our framework

def run_ours(args, rank, world, local, profile_hook=None):
    """Time ``args.steps`` sampling steps (device events, max over ranks) and the public
    pipeline end to end.  ``profile_hook(fn)``, when given, is called with a function that
    runs the steps instead of timing them (analysis tools; no bench line)."""
    from osp_next_b200 import ops
    from osp_next_b200.models.osp_next import OSPNextModel
    from osp_next_b200.parallel.cfg import CFGParallel
    from osp_next_b200.parallel.sp import attach_sp, build_sp_groups
    from osp_next_b200.pipelines.t2v import T2VInferencePipeline
    from osp_next_b200.schedulers.flow_matching import FlowMatchingScheduler

    cfg = PRESETS[args.model]
    dev = torch.device("cuda", local)
    torch.manual_seed(0)
    with torch.device(dev):
        model = OSPNextModel(**cfg)
    model = model.to(torch.bfloat16).eval()
    # norms / modulation stay fp32 (the reference's FSDP policy keeps norm params fp32)
    for n_, p in model.named_parameters():
        if "norm" in n_ or "modulation" in n_:
            p.data = p.data.float()
    # no text K/V cache: every timed step recomputes the cross-attention K/V like the reference
    cfg_size, ssp = layout_for(world)
    cfg_par = None
    if world > 1:
        rt = build_sp_groups(cfg["num_heads"], skiparse_sp_size=ssp, sp_size=1, cfg_size=cfg_size)
        attach_sp(model, rt)
        from osp_next_b200.parallel.sp_state import sp_state
        cfg_par = CFGParallel(sp_state.cfg_group) if cfg_size > 1 else None
        if ssp > 1 and args.exchange == "p2p":
            from osp_next_b200.parallel.sp import enable_p2p_exchange
            _, _, T, Hl, Wl = latent_shape(args)
            enable_p2p_exchange(model, 1, (T, Hl // 2, Wl // 2), dev)
    sched = FlowMatchingScheduler(num_inference_steps=STEPS_PER_VIDEO, guidance_scale=args.guidance,
                                  shift=args.shift)
    shape = latent_shape(args)
    g = torch.Generator().manual_seed(1234)
    text = torch.randn(1, cfg["text_len"], 4096, generator=g).to(torch.bfloat16)
    neg = torch.randn(1, cfg["text_len"], 4096, generator=g).to(torch.bfloat16)
    lat0 = torch.randn(shape, generator=g).to(torch.bfloat16)
    text_d, neg_d, lat_d = text.to(dev), neg.to(dev), lat0.to(dev)

    def device_steps(k):
        return sched.sample(model, lat_d.clone(), prompt_embeds=text_d, negative_prompt_embeds=neg_d,
                            cfg_parallel=cfg_par, max_steps=k)

    with torch.no_grad():
        device_steps(args.warmup)
        barrier_sync()
        if profile_hook is not None:
            profile_hook(lambda: device_steps(args.steps))
            barrier_sync()
            if getattr(getattr(model, "parallel", None), "p2p", None) is not None:
                model.parallel.p2p.close()
            return None
        clock = ClockSampler(local)
        clock.start()
        l0 = ops._ext.launch_count()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier_sync()
        ev0.record()
        out = device_steps(args.steps)
        ev1.record()
        barrier_sync()
        launches = ops._ext.launch_count() - l0
        clocks = clock.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms)
    finite = bool(torch.isfinite(out.float()).all())

    e2e = None
    if not args.no_e2e:
        pipe = T2VInferencePipeline(predictor=model, scheduler=sched)
        text_h, neg_h, lat_h = text.pin_memory(), neg.pin_memory(), lat0.pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in (text_h, neg_h, lat_h))
        barrier_sync()
        t0 = time.perf_counter()
        res = pipe(prompt_embeds=text_h, negative_prompt_embeds=neg_h, latents=lat_h, num_frames=args.frames,
                   height=args.height, width=args.width, device=dev, output_type="latent", cfg_parallel=cfg_par,
                   max_steps=args.steps)
        res_h = res.to("cpu")
        d2h = res_h.numel() * res_h.element_size()
        barrier_sync()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": round(e2e_s / args.steps * STEPS_PER_VIDEO, 3), "unit": "s/video",
               "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps,
               "note": "public T2VInferencePipeline call; inputs from pinned host, latent read back"}
    err = ops.ext().get_error(local, True)
    if getattr(getattr(model, "parallel", None), "p2p", None) is not None:
        model.parallel.p2p.close()
    return ms, launches, clocks, e2e, {"finite": finite, "device_error": err}


# ----------------------------------------------------------------------------- training

TRAIN_CONFIGS = {"14b": "configs/train/osp_14b.yaml", "1.3b": "configs/train/osp_1_3b.yaml",
                 "tiny": "configs/train/osp_tiny_cpu.yaml"}


def train_layout(world: int):
    """(fsdp, ssp) per GPU count for training: FSDP over every rank, SSP up to 4
    (8 GPUs = 2 SSP groups of 4 as data parallel, the reference's 14B layout)."""
    return world, min(world, 4)


def train_config(args, world, out_dir):
    from osp_next_b200.utils.config import load_config
    cfg = load_config(os.path.join(ROOT, TRAIN_CONFIGS[args.model]))
    fsdp, ssp = train_layout(world)
    cfg.update(output_dir=out_dir, training_iteration=10 ** 9, max_steps=args.warmup + args.steps,
               save_interval=10 ** 9, log_interval=1, fsdp_size=fsdp, skiparse_sp_size=ssp,
               use_skiparse_sequence_parallel=ssp > 1, sp_size=1, use_sequence_parallel=False,
               weight_dtype="bf16", gradient_checkpointing=True, seed=1024,
               fsdp_p2p_collectives=getattr(args, "fsdp_comm", "p2p") == "p2p",
               ssp_p2p_exchange=getattr(args, "exchange", "p2p") == "p2p")
    cfg["model_config"] = dict(cfg.get("model_config", {}), **{k: v for k, v in PRESETS[args.model].items()})
    cfg["model_config"].pop("pretrained_model_dir_or_checkpoint", None)
    if getattr(args, "quant", "none") == "hif8":
        cfg["model_config"].update(quant="hif8")
    if getattr(args, "loss_log", None):
        cfg["metrics_file"] = args.loss_log
    dc = dict(cfg.get("data_config", {}))
    dc.update(dataset_name="t2v_random_latent", num_workers=2, pin_memory=True, batch_size=1,
              dataset_config=dict(sample_height=args.height, sample_width=args.width,
                                  sample_num_frames=args.frames, text_max_length=PRESETS[args.model]["text_len"]))
    cfg["data_config"] = dc
    return cfg


def run_train(args, rank, world, local, impl):
    """Flow-matching training through the public trainer (``train/train_osp.py``): every
    step loads a synthetic latent/text batch from pinned host memory, runs the FSDP2 + SSP
    forward/backward with activation checkpointing, clips, AdamW, EMA, and reads the loss
    back.  tokens/s = tokens of all data-parallel groups / device step time (max over ranks)."""
    import tempfile
    sys.path.insert(0, os.path.join(ROOT, "train"))
    out_dir = tempfile.mkdtemp(prefix="osp_bench_train_")
    cfg = train_config(args, world, out_dir)
    rec = []
    clock = ClockSampler(local)

    def on_step(it, ms, tok):
        if it == args.warmup:
            clock.start()
        if it > args.warmup:
            rec.append((ms, tok, time.perf_counter()))

    t_first = [None]

    def on_step_wall(it, ms, tok):
        if it == args.warmup:
            t_first[0] = time.perf_counter()
        on_step(it, ms, tok)

    if impl == "reference":
        sys.path.insert(0, os.path.join(ROOT, "baseline"))
        import ref_harness
        if not os.path.isdir(os.path.join(ref_harness.REF_ROOT, "ospnext")):
            return {"metric": "train tokens/s", "impl": "reference", "unavailable": "reference not installed"}
        import ref_train
        ref_train.train(cfg, on_step_wall)
    else:
        import train_osp
        train_osp.main(cfg, on_step=on_step_wall)
    clocks = clock.stop()
    ms = max_over_ranks(sum(r[0] for r in rec) / len(rec))
    tok = rec[-1][1]
    wall = max_over_ranks((rec[-1][2] - t_first[0]) / len(rec))
    fsdp, ssp = train_layout(world)
    q = "" if args.quant == "none" else f" {args.quant}"
    return {"metric": f"train tokens/s OSP-Next-{args.model}{q} flow matching {args.frames}f "
                      f"{args.height}x{args.width}", "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak" if world > 4 else "strong",
            "dtype": "bf16", "impl": impl,
            "data": "synthetic (random-init weights, N(0,1) latents and text embeddings, logit-normal t)",
            "layout": {"fsdp_comm": args.fsdp_comm if impl == "ours" else "nccl"},
            "config": {"model": f"OSP-Next-{args.model}", "global_batch": max(1, world // ssp),
                       "seq_len": tokens(args), "parallelism": f"fsdp{fsdp}_ssp{ssp}_dp{max(1, world // ssp)}",
                       "activation_checkpointing": True, "optimizer": "AdamW + adaptive clip + EMA",
                       "l2": "no flush: per-step activations exceed the 126 MB L2"},
            "value": round(tok / (ms / 1000.0), 1), "ms_per_step": round(ms, 2), "vs_baseline": None,
            "clocks": clocks,
            "e2e": {"value": round(tok / wall, 1), "unit": "tokens/s",
                    "note": "host wall time per trainer step (pinned-host batch copy, loss read back)"}}


# ----------------------------------------------------------------------------- reference

def run_reference(args, rank, world, local):
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import ref_harness
    if not os.path.isdir(os.path.join(ref_harness.REF_ROOT, "ospnext")):
        return None, "reference not installed in baseline/_ref"
    fa2 = ref_harness.fa2_usable()
    osp, fm = ref_harness.import_reference(disable_compile=False, force_sdpa=not fa2)
    cfg = dict(PRESETS[args.model])
    dev = torch.device("cuda", local)
    if world > 1:
        from torch.distributed.device_mesh import init_device_mesh
        from ospnext.distributed.sp_state import sp_state
        ssp = min(world, 4)
        ul = world // ssp
        mesh = init_device_mesh("cuda", (1, ssp, ul), mesh_dim_names=("dp", "skiparse_sp", "sp"))
        gsp = mesh["skiparse_sp", "sp"]._flatten().get_group()
        full_size = math.gcd(cfg["num_heads"], world)
        full_mesh = init_device_mesh("cuda", (world // full_size, full_size), mesh_dim_names=("x", "full_sp"))
        sp_state.reset(global_sp_group=gsp, sp_group=mesh["sp"].get_group() if ul > 1 else None,
                       skiparse_sp_group=mesh["skiparse_sp"].get_group(),
                       full_sp_group=full_mesh["full_sp"].get_group())
    torch.manual_seed(0)
    with torch.device(dev):
        model = osp.OSPNextModel(**cfg)
    model = model.to(torch.bfloat16).eval()
    sched = fm.FlowMatchingScheduler(num_inference_steps=args.warmup, guidance_scale=args.guidance,
                                     shift=args.shift)
    shape = latent_shape(args)
    g = torch.Generator().manual_seed(1234)
    text = torch.randn(1, cfg["text_len"], 4096, generator=g).to(torch.bfloat16).to(dev)
    neg = torch.randn(1, cfg["text_len"], 4096, generator=g).to(torch.bfloat16).to(dev)
    lat = torch.randn(shape, generator=g).to(torch.bfloat16).to(dev)
    with torch.no_grad():
        sched.sample(model, lat.clone(), prompt_embeds=text, negative_prompt_embeds=neg)
        barrier_sync()
        sched.num_inference_steps = args.steps
        clock = ClockSampler(local)
        clock.start()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier_sync()
        ev0.record()
        sched.sample(model, lat.clone(), prompt_embeds=text, negative_prompt_embeds=neg)
        ev1.record()
        barrier_sync()
        clocks = clock.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    clocks["attention_backend"] = "flash_attn2" if fa2 else "sdpa"
    e2e = None
    if not args.no_e2e:
        e2e = reference_e2e(args, model, sched, text, neg, lat)
    return (ms, clocks, e2e), None


def reference_e2e(args, model, sched, text, neg, lat):
    """End to end through the reference's own code: its T2VInferencePipeline.prepare_latents
    (device copy + SP broadcast) and FlowMatchingScheduler.sample, with prompt embeddings and
    the initial latent copied from pinned host memory inside the timed region and the final
    latent read back.  The pipeline's ``__call__`` always VAE-decodes and draws its own noise,
    so its two denoising building blocks are called directly on the same inputs as ours."""
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    from ospnext.pipelines.t2v_pipeline import T2VInferencePipeline as RefPipeline
    pipe = RefPipeline(vae=None, tokenizer=None, text_encoder=None, predictor=model, scheduler=sched)
    text_h, neg_h, lat_h = text.cpu().pin_memory(), neg.cpu().pin_memory(), lat.cpu().pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (text_h, neg_h, lat_h))
    dev = lat.device
    sched.num_inference_steps = args.steps
    with torch.no_grad():
        barrier_sync()
        t0 = time.perf_counter()
        pe = text_h.to(dev, non_blocking=True)
        ne = neg_h.to(dev, non_blocking=True)
        latents = pipe.prepare_latents(lat_h.shape, generator=None, device=dev, dtype=pe.dtype, latents=lat_h)
        out = sched.sample(model=model, latents=latents, prompt_embeds=pe, negative_prompt_embeds=ne)
        out_h = out.to("cpu")
        barrier_sync()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
    d2h = out_h.numel() * out_h.element_size()
    return {"value": round(e2e_s / args.steps * STEPS_PER_VIDEO, 3), "unit": "s/video",
            "h2d_bytes_per_step": h2d // args.steps, "d2h_bytes_per_step": d2h // args.steps,
            "note": "reference T2VInferencePipeline.prepare_latents + FlowMatchingScheduler.sample; "
                    "inputs from pinned host, latent read back"}


# ----------------------------------------------------------------------------- main

def main():
    args = parse()
    # training also gathers CPU objects (loss logs, sampler state): gloo beside NCCL
    rank, world, local = init_dist(args.gpus, "cpu:gloo,cuda:nccl" if args.mode == "train" else "nccl")
    if args.mode == "train":
        if args.model == "14b" and world == 1:
            line = {"metric": "train tokens/s OSP-Next-14b", "n_gpus": 1, "impl": args.impl,
                    "unavailable": "14B AdamW training state (fp32 params, grads, moments, EMA: ~285 GB) "
                                   "does not fit one 180 GB GPU; needs FSDP over >= 2 GPUs"}
        else:
            line = run_train(args, rank, world, local, args.impl)
        if rank == 0:
            print(json.dumps(line))
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
        return
    cfg_size, ssp = layout_for(world)
    par = {1: "single", 2: "cfg2", 4: "cfg2_ssp2", 8: "cfg2_ssp4"}[world]
    if world >= 4 and args.impl == "ours":
        par += "_" + args.exchange
    base = {"metric": "sec/video OSP-Next-14B 81f 720P(padded 768x1280) 50-step CFG5 T2V",
            "unit": "s/video", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (random-init 14B weights, N(0,1) latents and 512x4096 text embeddings)",
            # the workload only (identical for both arms); the parallel layout is reported in "layout"
            "config": {"model": f"OSP-Next-{args.model}", "global_batch": 1, "seq_len": tokens(args),
                       "latent": list(latent_shape(args)), "steps_per_video": STEPS_PER_VIDEO,
                       "guidance_scale": args.guidance, "parallelism": f"{world}gpu_sequence_parallel",
                       "l2": "no flush: per-step activations (1.6 GB) exceed the 126 MB L2"}}
    if args.impl == "reference":
        res, why = run_reference(args, rank, world, local)
        if rank == 0:
            if res is None:
                print(json.dumps({"impl": "reference", "unavailable": why}))
            else:
                ms, clocks, e2e = res
                line = dict(base, impl="reference", value=round(ms * STEPS_PER_VIDEO / 1000, 3),
                            ms_per_step=round(ms, 2), vs_baseline=None, clocks=clocks, e2e=e2e,
                            layout=f"ssp{min(world, 4)}_ulysses{max(1, world // 4)}")
                print(json.dumps(line))
    else:
        ms, launches, clocks, e2e, extra = run_ours(args, rank, world, local)
        if rank == 0:
            val = ms * STEPS_PER_VIDEO / 1000.0
            line = dict(base, impl="ours", value=round(val, 3), ms_per_step=round(ms, 2),
                        vs_baseline=(None if BASELINE_SEC_PER_VIDEO is None else BASELINE_SEC_PER_VIDEO / val),
                        gpu_launches=launches, clocks=clocks, e2e=e2e, checks=extra, layout=par)
            print(json.dumps(line))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
