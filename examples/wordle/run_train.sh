#!/bin/bash
# Trainer for the wordle example over NUM_GPUS GPUs (data parallel, sharded optimizer state).
# SGLANG_URLS: comma-separated engine URLs started by serve.sh.
set -e
cd "$(dirname "$0")"
export SGLANG_URLS=${SGLANG_URLS:-http://127.0.0.1:30000}
export PYTORCH_CUDA_ALLOC_CONF=expandable_segments:True
exec torchrun --nproc-per-node ${NUM_GPUS:-1} --master-addr 127.0.0.1 --master-port ${MASTER_PORT:-29700} \
  train.py --model ${MODEL_PATH:-gpt-oss-20b} --run-dir ${RUN_DIR:-../../runs/wordle} "$@"
