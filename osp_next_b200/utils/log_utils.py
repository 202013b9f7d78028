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
