#!/bin/bash
# Rollout engine for the minesweeper example: one sglang-compatible server over TP_SIZE GPUs
# (tensor parallel under torchrun; rank 0 serves HTTP).  MODEL_PATH: preset name or checkpoint.
set -e
MODEL_PATH=${MODEL_PATH:-gpt-oss-20b}
TP_SIZE=${TP_SIZE:-1}
PORT=${PORT:-30000}
GPUS=${GPUS:-0}
export CUDA_VISIBLE_DEVICES=$GPUS
ARGS="--model $MODEL_PATH --port $PORT --lora-r ${LORA_R:-32} --lora-targets q_proj,k_proj,v_proj,o_proj,gate_up_proj,down_proj --max-running-requests 128 ${EXTRA_ARGS:-}"
if [ "$TP_SIZE" -gt 1 ]; then
  exec torchrun --nproc-per-node $TP_SIZE --master-addr 127.0.0.1 --master-port ${MASTER_PORT:-29600} \
    -m agent_factory_3_b200.engine.server $ARGS
else
  exec python -m agent_factory_3_b200.engine.server $ARGS
fi
