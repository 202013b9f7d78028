"""FSDP2 sharding with the reference's mixed-precision policy.

Reference: ospnext/distributed/fsdp2_wrapper.py:11-104 — ``fully_shard`` every
norm module with fp32 params, every main block with bf16 params and fp32
gradient reduction, then the root; HSDP when the mesh is 2-D; optional CPU
offload.  Parameter all-gather / gradient reduce-scatter run on NCCL inside
FSDP2 here; the optimizer step over the resulting fp32 shards is the fused
sm_100a AdamW kernel (:class:`osp_next_b200.parallel.optim.FusedAdamW`).
"""
from __future__ import annotations

import logging

import torch
import torch.distributed as dist
from torch.distributed.fsdp import CPUOffloadPolicy, MixedPrecisionPolicy, fully_shard


def _is_main():
    return not dist.is_initialized() or dist.get_rank() == 0


def FSDP2_mix_wrapper(model, dp_mesh=None, weight_dtype=torch.bfloat16, main_block_to_half=None,
                      blocks_to_float=None, blocks_to_output_float=None, reshard_after_forward=None,
                      cpu_offload=False):
    low = MixedPrecisionPolicy(param_dtype=weight_dtype, reduce_dtype=torch.float32, output_dtype=weight_dtype)
    high = MixedPrecisionPolicy(param_dtype=torch.float32, reduce_dtype=torch.float32, output_dtype=weight_dtype)
    full32 = MixedPrecisionPolicy(param_dtype=torch.float32, reduce_dtype=torch.float32, output_dtype=torch.float32)
    kw = {"reshard_after_forward": True if reshard_after_forward is None else reshard_after_forward,
          "mesh": dp_mesh}
    if cpu_offload:
        kw["offload_policy"] = CPUOffloadPolicy()
    for block in blocks_to_output_float or []:
        for m in model.modules():
            if isinstance(m, block):
                fully_shard(m, mp_policy=full32, **kw)
    for block in blocks_to_float or []:
        for m in model.modules():
            if isinstance(m, block) and any(p.numel() for p in m.parameters(recurse=False)):
                fully_shard(m, mp_policy=high, **kw)
    if main_block_to_half is not None:
        for m in model.modules():
            if isinstance(m, main_block_to_half):
                fully_shard(m, mp_policy=low, **kw)
    fully_shard(model, mp_policy=low, **kw)
    if _is_main():
        logging.info("FSDP2 sharding done")
    return model


def FSDP2_fp32_wrapper(model, dp_mesh=None, main_block=None, reshard_after_forward=None, cpu_offload=False):
    p = MixedPrecisionPolicy(param_dtype=torch.float32, reduce_dtype=torch.float32, output_dtype=torch.float32)
    kw = {"reshard_after_forward": True if reshard_after_forward is None else reshard_after_forward,
          "mesh": dp_mesh}
    if cpu_offload:
        kw["offload_policy"] = CPUOffloadPolicy()
    if main_block is not None:
        for m in model.modules():
            if isinstance(m, main_block):
                fully_shard(m, mp_policy=p, **kw)
    fully_shard(model, mp_policy=p, **kw)
    return model


def set_modules_to_forward_prefetch(blocks, num_to_forward_prefetch: int):
    """Explicit forward prefetch of the next N blocks (distributed/utils.py:23-32)."""
    for i, b in enumerate(blocks):
        if i >= len(blocks) - num_to_forward_prefetch:
            break
        b.set_modules_to_forward_prefetch([blocks[i + j] for j in range(1, num_to_forward_prefetch + 1)])


def set_modules_to_backward_prefetch(blocks, num_to_backward_prefetch: int):
    for i, b in enumerate(blocks):
        if i < num_to_backward_prefetch:
            continue
        b.set_modules_to_backward_prefetch([blocks[i - j] for j in range(1, num_to_backward_prefetch + 1)])
