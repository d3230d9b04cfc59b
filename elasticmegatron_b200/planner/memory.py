"""Device-memory estimate of a layout, and of a switch, from the layout functions alone (no GPU).

* state: the three arenas of a rank - parameters (model dtype), fp32 gradients (``main_grad``), fp32 optimizer
  ``[3, n]`` (master, exp_avg, exp_avg_sq of the rank's ZeRO shard) - exact, from ``planner/layout.py``;
* activations: an estimate of what one micro-batch keeps for the backward pass without recomputation, per
  transformer layer and token: the layer input and the norm outputs (3 h), the fused QKV output (h + 2 kv),
  the attention output (h), the fc1 output and the SwiGLU output (2 f' + f', f' = ffn / TP), stored in the model
  dtype, divided by TP where sequence parallelism shards them; under 1F1B the first stage holds PP micro-batches
  in flight; with full recompute only each layer's input is kept, plus one layer's set during its replay;
* switch: source and destination arenas coexist while the state moves (the source is released after).

The reference has no estimator; its release / rebuild machinery exists because several layouts do not fit at
once (training_state.py:199-311).
"""
from __future__ import annotations

from typing import Dict, Iterable, Optional

from ..config import ModelConfig, TrainConfig
from .layout import rank_layout


def _dtype_bytes(cfg: ModelConfig) -> int:
    return 4 if cfg.params_dtype == "fp32" else 2


def state_bytes(cfg: ModelConfig, strategy, rank: int, overlap_grad_reduce: bool = True,
                ddp_bucket_size: Optional[int] = None) -> Dict[str, int]:
    rl = rank_layout(cfg, strategy, rank, overlap_grad_reduce, ddp_bucket_size)
    n, opt_n = rl.param_numel, rl.opt_numel
    out = {"params": n * _dtype_bytes(cfg), "grads": n * 4, "optimizer": opt_n * 12}
    out["total"] = sum(out.values())
    return out


def activation_bytes(cfg: ModelConfig, strategy, micro_batch_size: int = 1, recompute: bool = False) -> int:
    tp, pp, cp = (strategy.tensor_model_parallel_size, strategy.pipeline_model_parallel_size,
                  strategy.context_parallel_size)
    h = cfg.hidden_size
    kv = cfg.num_query_groups * (h // cfg.num_attention_heads)
    f = (cfg.moe_ffn_hidden_size * cfg.moe_router_topk if cfg.num_experts else cfg.ffn_hidden_size)
    tokens = cfg.seq_length * micro_batch_size // cp
    seq_sharded = 5 * h if strategy.sequence_parallel else 5 * h * tp  # inputs, norms, attention output
    per_token = seq_sharded / tp + (h + 2 * kv) / tp + 3 * f / tp
    layers = cfg.num_layers // pp
    in_flight = pp  # 1F1B: the first stage holds PP micro-batches
    if recompute:
        # only each layer's input stays (sequence-sharded under SP), plus one layer's full set while it replays
        layer_input = h / tp if strategy.sequence_parallel else h
        return int((layer_input * layers * in_flight + per_token) * tokens * _dtype_bytes(cfg))
    return int(per_token * tokens * layers * in_flight * _dtype_bytes(cfg))


def layout_report(cfg: ModelConfig, strategy, train: Optional[TrainConfig] = None) -> Dict[str, int]:
    """Largest per-rank state + activation estimate over the strategy's ranks (bytes)."""
    train = train or TrainConfig()
    worst = None
    for r in range(strategy.world_size):
        st = state_bytes(cfg, strategy, r, train.overlap_grad_reduce, train.ddp_bucket_size)
        if worst is None or st["total"] > worst["total"]:
            worst = dict(st)
    worst["activations"] = activation_bytes(cfg, strategy, train.micro_batch_size, train.recompute)
    worst["peak"] = worst["total"] + worst["activations"]
    return worst


def switch_peak_bytes(cfg: ModelConfig, src, dst, train: Optional[TrainConfig] = None) -> int:
    """Largest per-rank state held during a switch (source and destination arenas together)."""
    train = train or TrainConfig()
    peak = 0
    for r in range(max(src.world_size, dst.world_size)):
        b = 0
        for s in (src, dst):
            if r < s.world_size:
                b += state_bytes(cfg, s, r, train.overlap_grad_reduce, train.ddp_bucket_size)["total"]
        peak = max(peak, b)
    return peak


def fits(cfg: ModelConfig, strategies: Iterable, device_bytes: int, train: Optional[TrainConfig] = None) -> Dict:
    """For each strategy: does training fit, and does every switch into it from the others fit."""
    strategies = list(strategies)
    out = {}
    for s in strategies:
        rep = layout_report(cfg, s, train)
        worst_switch = max((switch_peak_bytes(cfg, o, s, train) for o in strategies if o != s), default=0)
        out[str(s)] = {"train_peak": rep["peak"], "switch_peak": worst_switch,
                       "fits": rep["peak"] <= device_bytes and worst_switch <= device_bytes}
    return out
