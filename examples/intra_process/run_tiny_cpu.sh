#!/usr/bin/env bash
# The plumbing check without a GPU: tiny Llama (4 layers, hidden 512, 8 heads, SwiGLU 1376, vocab 32000,
# seq 512, micro-batch 2, global batch 8, Adam lr 3e-4, fp32) on 2 gloo ranks, switching DP2 -> TP2 -> PP2 -> DP2
# every 10 iterations, then the same run without switches, and the loss-continuity report.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
OUT="${OUT:-$HERE/logs}"
mkdir -p "$OUT"
COMMON=(--cpu --model tiny-llama --switch-every 10 --train-iters 40 --micro-batch-size 2 --global-batch-size 8
        --lr 3e-4 --lr-warmup-iters 0 --seed 0)
python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29662 \
    "$HERE/train_elastic.py" "${COMMON[@]}" --strategies ws2,ws2-tp2,ws2-pp2,ws2 > "$OUT/tiny_switch.log" 2>&1
python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29661 \
    "$HERE/train_elastic.py" "${COMMON[@]}" --strategies ws2 > "$OUT/tiny_base.log" 2>&1
PYTHONPATH="$HERE/../.." python -m elasticmegatron_b200.tools.loss_curve "$OUT/tiny_base.log" "$OUT/tiny_switch.log"
