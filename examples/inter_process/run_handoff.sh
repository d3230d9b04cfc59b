#!/usr/bin/env bash
# Scale a running job from 8 to 4 GPUs (and from DP8 to TP2*DP2) by handing its state to a new job.
# The old job starts the successor itself at --handoff-at; both print Megatron-style iteration lines.
#   bash examples/inter_process/run_handoff.sh
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
NPROC="${NPROC:-8}"
NEW_NPROC="${NEW_NPROC:-4}"
MODEL="${MODEL:-llama2-7b}"
PORT="${MASTER_PORT:-29500}"
NEW_PORT="${NEW_MASTER_PORT:-29700}"
python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NPROC" --master-addr 127.0.0.1 --master-port "$PORT" \
    "$HERE/train_handoff.py" --model "$MODEL" --strategy "ws$NPROC" --successor-strategy "ws$NEW_NPROC-tp2" \
    --successor-nproc "$NEW_NPROC" --successor-port "$NEW_PORT" --handoff-at 5 --train-iters 20 \
    --global-batch-size 32 --wait-successor "$@"
