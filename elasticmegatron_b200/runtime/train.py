"""One optimizer step under any strategy.

``train_step(ts, data_iter)`` is the public training call: it pulls this rank's micro-batches (pinned host
memory), copies each to the device asynchronously, runs the strategy's schedule (no pipelining or 1F1B),
finishes DP gradient reduction, takes the distributed Adam step, all-gathers parameters and advances the LR
schedule by ``num_microbatches * MBS * DP`` samples (Megatron's train_step, which the reference's example
loops call; examples/intra_process/training_011.py:837-928).
"""
from __future__ import annotations

from typing import Dict, Iterator, List, Optional

import torch
import torch.distributed as dist

from ..parallel.pipeline import StepContext, get_forward_backward_func
from .data import num_microbatches


def _act_shape(ts) -> tuple:
    cfg, s = ts.cfg, ts.strategy
    tokens = cfg.seq_length // s.context_parallel_size * ts.train_cfg.micro_batch_size
    if s.sequence_parallel and s.tensor_model_parallel_size > 1:
        tokens //= s.tensor_model_parallel_size
    return (tokens, cfg.hidden_size)


def train_step(ts, data_iter: Iterator, hetero_dp: Optional[bool] = None, return_loss: bool = True) -> Dict:
    ps, tc, cfg = ts.ps, ts.train_cfg, ts.cfg
    s = ts.strategy
    from .hetero_dp import hetero_alignment, hetero_dp_enabled, process_outputs

    if hetero_dp is None:
        hetero_dp = hetero_dp_enabled()
    n_mb = num_microbatches(tc.global_batch_size, tc.micro_batch_size, s.data_parallel_size, ps.dp_rank, hetero_dp,
                            hetero_alignment() if hetero_dp else 1)
    dev = ts.device
    needs_data = ps.is_first_stage or ps.is_last_stage
    host = [next(data_iter) for _ in range(n_mb)] if needs_data else [(None, None)] * n_mb
    batches = []
    for ids, lab in host:
        if ids is None:
            batches.append((None, None))
        else:
            batches.append((ids.to(dev, non_blocking=True), lab.to(dev, non_blocking=True)))
    ts.ddp.zero_grad()
    # Every rank scales its token-loss sum by DP*CP / (GBS * seq): after the optimizer's 1/(DP*CP) gradient
    # average this is the gradient of the global mean token loss, also when DP ranks run different numbers
    # of micro-batches (hetero-DP).
    loss_scale = (s.data_parallel_size * s.context_parallel_size) / (tc.global_batch_size * cfg.seq_length)
    ctx = StepContext(ts.stage, ps, ts.ddp, n_mb, _act_shape(ts), ts.param_dtype, dev, loss_scale,
                      lambda i: batches[i])
    fb = get_forward_backward_func(s.pipeline_model_parallel_size)
    loss_sums = fb(ctx)
    ts.ddp.finish_grad_sync()
    ok, gnorm = ts.optimizer.step()
    ts.ddp.start_param_sync(overlap=tc.overlap_param_gather)
    ts.opt_param_scheduler.step(n_mb * tc.micro_batch_size * s.data_parallel_size if not hetero_dp
                                else tc.global_batch_size)
    out = {"grad_norm": gnorm, "num_microbatches": n_mb, "update_successful": ok}
    if return_loss:
        if hetero_dp and ps.is_last_stage and loss_sums:
            loss_sums = process_outputs(loss_sums)
        out["loss"] = reduce_loss(ts, loss_sums)
    if ts.pool.guard:
        from .memory import check_guards

        check_guards("train_step")
    return out


def reduce_loss(ts, loss_sums: List[torch.Tensor]) -> float:
    """Mean token loss of the global batch, identical on every rank of the strategy (one all-reduce)."""
    ps, tc, cfg = ts.ps, ts.train_cfg, ts.cfg
    if ps.is_last_stage and ps.tp_rank == 0 and loss_sums:
        t = torch.stack(loss_sums).sum().float().reshape(1)
    else:
        t = torch.zeros(1, dtype=torch.float32, device=ts.device)
    g = ps.group("world")
    if g is not None and dist.get_world_size(g) > 1:
        dist.all_reduce(t, group=g)
    loss = float(t.item()) / (tc.global_batch_size * cfg.seq_length)
    if t.is_cuda:
        from ..ops.native import check_device_errors

        check_device_errors()
    return loss
