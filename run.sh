#!/usr/bin/env bash
# Launcher (reference run.sh): maps shell flags to train.py flags and starts one process per GPU.
#   bash run.sh --task train --model_path TinyLlama/TinyLlama_v1.1 --gpus 8 [extra train.py flags]
set -euo pipefail
TASK=train; MODEL=TinyLlama/TinyLlama_v1.1; BATCH=1024; MIC=1; LR=5e-5; CTX=2048; SEED=4321
GPUS=${GPUS:-1}; MASTER=${MASTER:-127.0.0.1}; PORT=${PORT:-18010}; NNODES=${NNODES:-1}; NODE_RANK=${NODE_RANK:-0}
EXTRA=()
while [[ $# -gt 0 ]]; do
  case "$1" in
    --task) TASK="$2"; shift 2;;
    --model_path) MODEL="$2"; shift 2;;
    --batch_size) BATCH="$2"; shift 2;;
    --micro_batch_size) MIC="$2"; shift 2;;
    --learning_rate) LR="$2"; shift 2;;
    --context_length) CTX="$2"; shift 2;;
    --random_seed) SEED="$2"; shift 2;;
    --gpus) GPUS="$2"; shift 2;;
    --master_addr) MASTER="$2"; shift 2;;
    --master_port) PORT="$2"; shift 2;;
    --nnodes) NNODES="$2"; shift 2;;
    --node_rank) NODE_RANK="$2"; shift 2;;
    *) EXTRA+=("$1"); shift;;
  esac
done
cd "$(dirname "$0")"
exec python -m torch.distributed.run --nnodes "$NNODES" --node-rank "$NODE_RANK" \
  --nproc-per-node "$GPUS" --master-addr "$MASTER" --master-port "$PORT" train.py \
  --task "$TASK" --model_path "$MODEL" --batch_size "$BATCH" --micro_batch_size "$MIC" \
  --learning_rate "$LR" --context_length "$CTX" --random_seed "$SEED" --weight_decay 1e-2 \
  --train_ratio 0.999 --eval_steps 1000 --save_steps 100 "${EXTRA[@]}"
