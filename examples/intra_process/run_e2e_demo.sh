#!/usr/bin/env bash
# Dense Llama-style model, one 8-GPU node, online switches between strategies every 2 iterations.
# Analogue of the reference's run_e2e_demo.sh (model, seq 4096, MBS 1, GBS 32, ZeRO-1, bf16, mock data).
#   NPROC=8 MODEL=llama2-7b bash examples/intra_process/run_e2e_demo.sh
#   MODEL=demo-tiny bash examples/intra_process/run_e2e_demo.sh   # the reference demo's own default model
#                                                                 # (4 layers, hidden 4096, LayerNorm)
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
NPROC="${NPROC:-8}"
MODEL="${MODEL:-llama2-7b}"
LAYERS="${LAYERS:-}"
PORT="${MASTER_PORT:-29500}"
ITERS="${TRAIN_ITERS:-20}"
STRATEGIES="${STRATEGIES:-}"   # e.g. ws8,ws2-tp2,ws4,ws2 (default: the reference's demo schedule)
GBS="${GBS:-32}"
if [ "${SCHEDULE:-}" = "tp-sweep" ]; then
  # TP8 -> TP4*DP2 -> TP2*PP2*DP2 -> TP1*DP8 on 8 GPUs, global batch 128 (SP on whenever TP > 1)
  STRATEGIES="ws8-tp8,ws8-tp4,ws8-tp2-pp2,ws8"
  GBS=128
fi
LOG_DIR="${LOG_DIR:-$HERE/logs}"
mkdir -p "$LOG_DIR"
export CUDA_DEVICE_MAX_CONNECTIONS="${CUDA_DEVICE_MAX_CONNECTIONS:-1}"
ARGS=(--model "$MODEL" --train-iters "$ITERS" --switch-every 2 --micro-batch-size 1 --global-batch-size "$GBS"
      --lr 3e-4 --min-lr 3e-5 --lr-warmup-iters 2 --overlap-grad-reduce)
[ -n "$LAYERS" ] && ARGS+=(--layers "$LAYERS")
[ -n "$STRATEGIES" ] && ARGS+=(--strategies "$STRATEGIES")
python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NPROC" --master-addr 127.0.0.1 --master-port "$PORT" \
    "$HERE/train_elastic.py" "${ARGS[@]}" "$@" 2>&1 | tee "$LOG_DIR/e2e_demo_$(date +%Y%m%d_%H%M%S).log"
