#!/usr/bin/env bash
# 8-GPU flow-matching training (reference: scripts/train/gpu/train_osp_14b.sh)
torchrun --nnodes=${NNODES:-1} --nproc-per-node ${NPROC_PER_NODE:-8} --master-addr ${MASTER_ADDR:-127.0.0.1} \
  --master-port ${MASTER_PORT:-29513} train/train_osp.py --config ${CONFIG:-configs/train/osp_14b.yaml}
