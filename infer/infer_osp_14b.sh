#!/usr/bin/env bash
# 8-GPU T2V inference (reference: scripts/infer/gpu/infer_osp_14b.sh)
NPROC=${NPROC_PER_NODE:-8}
torchrun --nnodes=${NNODES:-1} --nproc-per-node $NPROC --master-addr ${MASTER_ADDR:-127.0.0.1} \
  --master-port ${MASTER_PORT:-29512} infer/infer_osp.py --config ${CONFIG:-configs/infer/osp_14b.yaml}
