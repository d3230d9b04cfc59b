#!/usr/bin/env bash
# Mixtral-style MoE (8 experts, top-2, aux loss 1e-2, GQA, rope base 1e6), 2 layers, EP switches online.
# Analogue of the reference's run_moe.sh (EP4, SP on, ZeRO-1, full activation recompute).
#   NPROC=8 bash examples/intra_process/run_moe.sh
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
NPROC="${NPROC:-8}"
PORT="${MASTER_PORT:-29500}"
ITERS="${TRAIN_ITERS:-20}"
LOG_DIR="${LOG_DIR:-$HERE/logs}"
mkdir -p "$LOG_DIR"
STRATEGIES="${STRATEGIES:-ws${NPROC}-ep4,ws${NPROC}-tp2-ep4-etp1,ws${NPROC}-ep8,ws${NPROC}-ep2}"  # ETP stays 1 (experts are not TP-split)
python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NPROC" --master-addr 127.0.0.1 --master-port "$PORT" \
    "$HERE/train_elastic.py" --model mixtral-8x7b --layers 2 --train-iters "$ITERS" --switch-every 2 \
    --micro-batch-size 1 --global-batch-size 32 --strategies "$STRATEGIES" --recompute "$@" \
    2>&1 | tee "$LOG_DIR/moe_$(date +%Y%m%d_%H%M%S).log"
