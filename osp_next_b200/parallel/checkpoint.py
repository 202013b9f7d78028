"""Checkpoint save / resume in the reference's directory layout.

Reference: ospnext/distributed/checkpoint.py:24-352::

    {output_dir}/iter_{:09d}/model_state_dict.pt          full fp32 state dict (rank 0)
                             ema_model_state_dict.pt
                             optim_state_dict.pt
                             random_states/rank_{:06d}.pkl
                             dataloader_states/rank_{:06d}.pkl
                             adaptive_grad_clip_states.pt

Full state dicts are gathered with ``torch.distributed.checkpoint.state_dict``
(works for FSDP2 DTensors and plain modules) and loaded with
``broadcast_from_rank0``.  Addition: an iteration directory is written under a
temporary name and renamed when complete, so a crash never leaves a partial
checkpoint that resume would pick up (resume = newest complete ``iter_*``).
"""
from __future__ import annotations

import os
import pickle
import re
import shutil
from typing import Optional

import torch
import torch.distributed as dist
from torch.distributed.checkpoint.state_dict import (StateDictOptions, get_model_state_dict,
                                                     get_optimizer_state_dict, set_model_state_dict,
                                                     set_optimizer_state_dict)

from ..utils.random_utils import get_rng_state, set_rng_state

PREFIX = "iter_"
MODEL_CHECKPOINT = "model_state_dict.pt"
OPTIM_CHECKPOINT = "optim_state_dict.pt"
RNG_DIR = "random_states"
DATALOADER_DIR = "dataloader_states"


def _rank():
    return dist.get_rank() if dist.is_initialized() else 0


def _barrier():
    if dist.is_initialized():
        dist.barrier()


def get_latest_checkpoint_folder(root: str) -> int:
    """Newest complete iteration number under ``root`` (0 when none)."""
    if not root or not os.path.isdir(root):
        return 0
    its = [int(m.group(1)) for d in os.listdir(root) if (m := re.fullmatch(PREFIX + r"(\d{9})", d))]
    its = [i for i in its if os.path.exists(os.path.join(root, f"{PREFIX}{i:09d}", MODEL_CHECKPOINT))]
    return max(its) if its else 0


def load_full_state_dict(path: str) -> dict:
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file
        return load_file(path, device="cpu")
    return torch.load(path, mmap=True, weights_only=True, map_location="cpu")


class Checkpointer:
    def __init__(self, folder: Optional[str] = None, dcp_api: bool = True):
        self.folder = folder
        self.save_root_dir = folder
        self.dcp_api = dcp_api
        self._last_training_iteration = get_latest_checkpoint_folder(folder) if folder else 0

    @property
    def last_training_iteration(self) -> int:
        return self._last_training_iteration

    def iter_dir(self, it: int) -> str:
        return os.path.join(self.save_root_dir, f"{PREFIX}{it:09d}")

    # ------------------------------------------------------------------ model
    def load_state_dict(self, model: torch.nn.Module, full_sd: dict, strict: bool = False):
        own = set(model.state_dict().keys())
        unexpected = [k for k in full_sd if k not in own]
        missing = [k for k in own if k not in full_sd]
        sd = {k: v for k, v in full_sd.items() if k in own}
        set_model_state_dict(model, sd, options=StateDictOptions(full_state_dict=True, strict=strict,
                                                                 broadcast_from_rank0=False))
        if _rank() == 0 and (missing or unexpected):
            print("missing_keys", missing[:16], "... total", len(missing))
            print("unexpected_keys", unexpected[:16], "... total", len(unexpected))
        return missing, unexpected

    def load_model_from_path(self, model, model_path: str):
        return self.load_state_dict(model, load_full_state_dict(model_path))

    def load_model(self, model, ema: bool = False):
        name = f"ema_{MODEL_CHECKPOINT}" if ema else MODEL_CHECKPOINT
        p = os.path.join(self.iter_dir(self.last_training_iteration), name)
        if os.path.exists(p):
            self.load_state_dict(model, load_full_state_dict(p))
            return True
        return False

    def load_optim(self, model, opt):
        p = os.path.join(self.iter_dir(self.last_training_iteration), OPTIM_CHECKPOINT)
        if not os.path.exists(p):
            return False
        sd = torch.load(p, map_location="cpu", weights_only=False)
        set_optimizer_state_dict(model, opt, sd, options=StateDictOptions(full_state_dict=True))
        return True

    def load_rng(self):
        p = os.path.join(self.iter_dir(self.last_training_iteration), RNG_DIR, f"rank_{_rank():06d}.pkl")
        if os.path.exists(p):
            with open(p, "rb") as f:
                set_rng_state(pickle.load(f))

    def load_dataloader(self, dataloader):
        p = os.path.join(self.iter_dir(self.last_training_iteration), DATALOADER_DIR, f"rank_{_rank():06d}.pkl")
        if os.path.exists(p) and hasattr(dataloader, "load_state_dict"):
            with open(p, "rb") as f:
                dataloader.load_state_dict(pickle.load(f))

    # ------------------------------------------------------------------ save
    def save(self, it: int, model, optimizer=None, ema=None, dataloader=None, clipper=None, extra: dict = None):
        final = self.iter_dir(it)
        tmp = final + ".tmp"
        if _rank() == 0:
            shutil.rmtree(tmp, ignore_errors=True)
            os.makedirs(os.path.join(tmp, RNG_DIR), exist_ok=True)
            os.makedirs(os.path.join(tmp, DATALOADER_DIR), exist_ok=True)
        _barrier()
        opts = StateDictOptions(full_state_dict=True, cpu_offload=True)
        msd = get_model_state_dict(model, options=opts)
        if _rank() == 0:
            torch.save(msd, os.path.join(tmp, MODEL_CHECKPOINT))
        del msd
        if ema is not None:
            ema.store(model)
            ema.ema_copy_to_model(model)
            esd = get_model_state_dict(model, options=opts)
            ema.restore(model)
            if _rank() == 0:
                torch.save(esd, os.path.join(tmp, f"ema_{MODEL_CHECKPOINT}"))
            del esd
        if optimizer is not None:
            osd = get_optimizer_state_dict(model, optimizer, options=opts)
            if _rank() == 0:
                torch.save(osd, os.path.join(tmp, OPTIM_CHECKPOINT))
            del osd
        _barrier()
        with open(os.path.join(tmp, RNG_DIR, f"rank_{_rank():06d}.pkl"), "wb") as f:
            pickle.dump(get_rng_state(), f)
        if dataloader is not None and hasattr(dataloader, "state_dict"):
            with open(os.path.join(tmp, DATALOADER_DIR, f"rank_{_rank():06d}.pkl"), "wb") as f:
                pickle.dump(dataloader.state_dict(), f)
        if clipper is not None and _rank() == 0:
            clipper.save(tmp)
        if extra and _rank() == 0:
            torch.save(extra, os.path.join(tmp, "extra_state.pt"))
        _barrier()
        if _rank() == 0:
            shutil.rmtree(final, ignore_errors=True)
            os.replace(tmp, final)
        _barrier()
        self._last_training_iteration = it
        return final
