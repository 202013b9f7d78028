"""OSP-Next on B200: text-to-video Skiparse DiT framework written for sm_100a.

Layer map (top to bottom):
  train/, infer/                      entry points (YAML config → driver)
  pipelines/, schedulers/, rl/        T2V sampling, flow matching, Mix-GRPO
  models/                             OSP-Next DiT (Skiparse-2D), Wan DiT, T5, VAE, LoRA, HiF8
  parallel/                           SSP / Ulysses / CFG-parallel layouts, FSDP, EMA, checkpoints
  ops/                                sm_100a CUDA kernels (tcgen05 GEMM + attention, fused elementwise)
  utils/, data/, rewards/             logging, clipping, caches, datasets, reward models
"""
__version__ = "0.1.0"
