#!/usr/bin/env bash
# Inter-process scale-down and scale-up, 8 -> 4 -> 8 GPUs (Llama-3 8B, seq 8192, global batch 64): the first job
# trains on 8 GPUs with two Group-ZeRO optimizer instances, hands its state to a new 4-GPU job (the replicas are
# dropped), which later hands it to a new 8-GPU job (the replicas are rebuilt).  Each job starts the next one
# itself; every job prints Megatron-style iteration lines.
#   bash examples/inter_process/run_handoff.sh
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
NPROC="${NPROC:-8}"
MODEL="${MODEL:-llama3-8b}"
CHAIN="${CHAIN:-ws8-inst2,ws4,ws8-inst2}"
PORT="${MASTER_PORT:-29500}"
NEW_PORT="${NEW_MASTER_PORT:-29700}"
python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NPROC" --master-addr 127.0.0.1 --master-port "$PORT" \
    "$HERE/train_handoff.py" --model "$MODEL" --seq-length "${SEQ:-8192}" --chain "$CHAIN" \
    --successor-port "$NEW_PORT" --handoff-at "${HANDOFF_EVERY:-5}" --train-iters "${TRAIN_ITERS:-20}" \
    --global-batch-size "${GBS:-64}" --wait-successor "$@"
