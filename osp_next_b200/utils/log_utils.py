"""Rank-aware logging (reference: ospnext/utils/log_utils.py:1-26)."""
import logging
import os
import sys

import torch
import torch.distributed as dist

_LOGGER = None


def get_logger(name: str = "osp_next_b200") -> logging.Logger:
    global _LOGGER
    if _LOGGER is None:
        logging.basicConfig(
            level=logging.INFO,
            format="[%(asctime)s] %(levelname)s %(message)s",
            datefmt="%Y-%m-%d %H:%M:%S",
            stream=sys.stdout,
        )
        _LOGGER = logging.getLogger(name)
    return _LOGGER


def _rank() -> int:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank()
    return int(os.environ.get("RANK", "0"))


def log_on_main_process(logger: logging.Logger, msg: str) -> None:
    if _rank() == 0:
        logger.info(msg)


def verify_min_gpu_count(min_gpus: int = 2) -> bool:
    return torch.cuda.is_available() and torch.cuda.device_count() >= min_gpus


class MetricsLogger:
    """Step metrics to a JSONL file and, when the ``wandb`` package is importable and
    ``use_wandb`` is set, to a wandb run (reference: train_osp.py:110-119, 514-528;
    train_osp_RL.py:1283-1383).  Only rank 0 writes; other ranks' calls are no-ops."""

    def __init__(self, path: str = None, use_wandb: bool = False, project: str = "osp_next_b200",
                 run_name: str = None, config: dict = None):
        self.path = path
        self.enabled = _rank() == 0
        self.wandb = None
        if self.enabled and path:
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        if self.enabled and use_wandb:
            try:
                import wandb
                self.wandb = wandb
                if wandb.run is None:
                    wandb.init(project=project, name=run_name, config=config or {})
            except ImportError:
                get_logger().warning("use_wandb is set but the wandb package is not installed; JSONL only")

    def log(self, record: dict, step: int = None) -> None:
        if not self.enabled:
            return
        import json
        rec = {k: (float(v) if hasattr(v, "item") and getattr(v, "ndim", 0) == 0 else v) for k, v in record.items()}
        if step is not None:
            rec.setdefault("step", step)
        if self.path:
            with open(self.path, "a") as f:
                f.write(json.dumps(rec, default=float) + "\n")
        if self.wandb is not None:
            self.wandb.log({k: v for k, v in rec.items() if isinstance(v, (int, float))}, step=step)

    def close(self) -> None:
        if self.wandb is not None and self.wandb.run is not None:
            self.wandb.finish()
