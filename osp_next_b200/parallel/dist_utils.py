"""Process-group setup and tensor gather/broadcast helpers.

Reference: ospnext/distributed/utils.py:10-163 — ``cpu:gloo,cuda:nccl`` init,
gather/broadcast of tensor lists with shape/dtype headers, send/recv of videos
to rank 0.  The process-group timeout defaults to 600 s (the reference uses
3600 s) so a missing rank ends collectives with an error instead of waiting.
"""
from __future__ import annotations

import datetime
import os
from typing import List, Optional

import torch
import torch.distributed as dist

_DTYPES = [torch.float32, torch.float16, torch.bfloat16, torch.uint8, torch.int32, torch.int64, torch.bool]


def setup_distributed_env(backend: Optional[str] = None, timeout_s: int = 600):
    if dist.is_initialized():
        return
    if "RANK" not in os.environ:
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        os.environ.setdefault("LOCAL_RANK", "0")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
    if torch.cuda.is_available():
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        backend = backend or "cpu:gloo,cuda:nccl"
    else:
        backend = backend or "gloo"
    dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))


def cleanup_distributed_env():
    if dist.is_initialized():
        dist.destroy_process_group()


def _dev(group):
    if dist.get_backend(group) == "gloo":
        return torch.device("cpu")
    return torch.device("cuda", torch.cuda.current_device())


def gather_data_from_all_ranks(data: torch.Tensor, dim: int = 0, group=None) -> torch.Tensor:
    """All-gather equal-shaped tensors and concatenate along ``dim`` (0-dim inputs become [1])."""
    if not dist.is_initialized():
        return data.reshape(-1) if data.dim() == 0 else data
    d = data.reshape(1) if data.dim() == 0 else data.contiguous()
    out = [torch.empty_like(d) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, d, group=group)
    return torch.cat(out, dim=dim)


def broadcast_tensor_list(tensors: Optional[List[torch.Tensor]], src: int, group=None, device=None) -> List[torch.Tensor]:
    """Broadcast a list of tensors with a count/ndim/shape/dtype header (utils.py:53-99)."""
    device = device or _dev(group)
    rank = dist.get_rank()
    if rank == src:
        hdr = [len(tensors)]
        for t in tensors:
            hdr += [t.dim(), _DTYPES.index(t.dtype)] + list(t.shape)
        h = torch.tensor([len(hdr)] + hdr, dtype=torch.int64, device=device)
        n = torch.tensor([h.numel()], dtype=torch.int64, device=device)
    else:
        n = torch.zeros(1, dtype=torch.int64, device=device)
    dist.broadcast(n, src=src, group=group)
    if rank != src:
        h = torch.zeros(int(n.item()), dtype=torch.int64, device=device)
    dist.broadcast(h, src=src, group=group)
    hl = h.tolist()[1:]
    cnt, pos, out = hl[0], 1, []
    for i in range(cnt):
        nd, dt = hl[pos], _DTYPES[hl[pos + 1]]
        shape = hl[pos + 2: pos + 2 + nd]
        pos += 2 + nd
        buf = tensors[i].to(device).contiguous() if rank == src else torch.empty(shape, dtype=dt, device=device)
        dist.broadcast(buf, src=src, group=group)
        out.append(buf)
    return out


def gather_tensor_list_to_one(tensors: List[torch.Tensor], dst: int = 0, group=None) -> Optional[List[torch.Tensor]]:
    """Send every rank's list of tensors to ``dst`` (point-to-point, utils.py:101-163)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    device = _dev(group)
    if rank == dst:
        result = list(tensors)
        for r in range(world):
            if r == dst:
                continue
            src = dist.get_global_rank(group, r) if group is not None else r
            n = torch.zeros(1, dtype=torch.int64, device=device)
            dist.recv(n, src=src, group=group)
            for _ in range(int(n.item())):
                meta = torch.zeros(8, dtype=torch.int64, device=device)
                dist.recv(meta, src=src, group=group)
                nd, dt = int(meta[0]), _DTYPES[int(meta[1])]
                shape = meta[2:2 + nd].tolist()
                buf = torch.empty(shape, dtype=dt, device=device)
                dist.recv(buf, src=src, group=group)
                result.append(buf.cpu())
        return result
    dst_g = dist.get_global_rank(group, dst) if group is not None else dst
    dist.send(torch.tensor([len(tensors)], dtype=torch.int64, device=device), dst=dst_g, group=group)
    for t in tensors:
        assert t.dim() <= 6
        meta = torch.zeros(8, dtype=torch.int64, device=device)
        meta[0], meta[1] = t.dim(), _DTYPES.index(t.dtype)
        meta[2:2 + t.dim()] = torch.tensor(list(t.shape))
        dist.send(meta, dst=dst_g, group=group)
        dist.send(t.to(device).contiguous(), dst=dst_g, group=group)
    return None
