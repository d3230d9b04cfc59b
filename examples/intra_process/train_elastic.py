"""Intra-process elastic training: one job switches parallel strategies online while it trains.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 examples/intra_process/train_elastic.py \
        --model llama2-7b --strategies ws8,ws2-tp2,ws4,ws2,ws8 --switch-every 2 --train-iters 20

Every process of the job stays alive for the whole run.  Strategy ``k`` uses ranks ``0..ws_k-1``; ranks outside
it idle (they still enter ``reshard`` so that they can hand over or receive state).  Every ``--switch-every``
iterations all ranks meet at a host barrier and switch to the next strategy of the list (cyclically); the data
stream resumes at the consumed-sample count, so the loss curve continues as if nothing happened.

This is the analogue of the reference's Megatron-0.11 example loop (examples/intra_process/training_011.py:
strategy list :100-133, manager set-up :140-143, reshard check :145-153, loop hook :1520-1555), written against
this framework's own training core.  Runs on GPUs (NCCL) or, with ``--cpu``, on gloo ranks.

Log lines use Megatron's format, so ``python -m elasticmegatron_b200.tools.loss_curve`` reads them.
"""
from __future__ import annotations

import argparse
import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))  # run from a checkout

def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-llama", help="preset name (config.PRESETS)")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--seq-length", type=int, default=None)
    ap.add_argument("--num-experts", type=int, default=None, help="override the preset's expert count (MoE)")
    ap.add_argument("--moe-ffn", type=int, default=None, help="override the experts' ffn size")
    ap.add_argument("--strategies", default=None,
                    help="comma list of strategy specs, e.g. ws8,ws2-tp2,ws4,ws2 (default: the reference's demo "
                         "schedule scaled to the job size)")
    ap.add_argument("--switch-every", type=int, default=2)
    ap.add_argument("--train-iters", type=int, default=20)
    ap.add_argument("--micro-batch-size", type=int, default=1)
    ap.add_argument("--global-batch-size", type=int, default=32)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--min-lr", type=float, default=3e-5)
    ap.add_argument("--lr-warmup-iters", type=int, default=2)
    ap.add_argument("--engine", default=None, choices=[None, "native", "torch", "reference"])
    ap.add_argument("--overlap-grad-reduce", action="store_true")
    ap.add_argument("--recompute", action="store_true",
                    help="recompute every transformer layer's activations in backward (full, one layer each)")
    ap.add_argument("--cp-comm-type", default="all_gather", choices=["all_gather", "p2p", "a2a"],
                    help="context parallelism: gather K/V over the CP group, pass it round a ring, or all-to-all "
                         "to a query-group split (Ulysses)")
    ap.add_argument("--save", default=None, help="checkpoint directory written at the end")
    ap.add_argument("--save-around-reshard", action="store_true",
                    help="write before_reshard/ and after_reshard/ checkpoints at every switch (for compare_ckpt)")
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--cpu", action="store_true", help="gloo ranks on CPU (fp32)")
    return ap.parse_args(argv)


def default_schedule(world: int):
    """The reference's demo schedule 8 -> (ws2, TP2) -> (ws4, TP1) -> (ws2, TP1) -> 8, scaled to ``world``."""
    out = [f"ws{world}"]
    if world >= 2:
        out.append("ws2-tp2")
    if world >= 4:
        out.append(f"ws{world // 2}")
    if world >= 2:
        out.append("ws2")
    return out


def main(argv=None):
    a = parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and not a.cpu
    if use_cuda:
        torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    dist.init_process_group("nccl" if use_cuda else "gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=600),
                            **({"device_id": torch.device("cuda", local)} if use_cuda else {}))

    from elasticmegatron_b200 import ElasticMegatronManager
    from elasticmegatron_b200.config import Args, TrainConfig, get_args, preset, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState
    from elasticmegatron_b200.utils.logging import log_json

    over = {"max_tensor_parallel_size": 8}
    if a.layers:
        over["num_layers"] = a.layers
    if a.seq_length:
        over["seq_length"] = a.seq_length
    if a.num_experts:
        over["num_experts"] = a.num_experts
    if a.moe_ffn:
        over["moe_ffn_hidden_size"] = a.moe_ffn
    over["params_dtype"] = "bf16" if use_cuda else "fp32"  # the CUDA kernels are bf16; CPU ranks run fp32
    cfg = preset(a.model, **over)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=a.micro_batch_size,
                                               global_batch_size=a.global_batch_size, lr=a.lr, min_lr=a.min_lr,
                                               lr_warmup_iters=a.lr_warmup_iters, train_iters=a.train_iters,
                                               overlap_grad_reduce=a.overlap_grad_reduce,
                                               cp_comm_type=a.cp_comm_type, recompute=a.recompute)))
    specs = a.strategies.split(",") if a.strategies else default_schedule(world)
    strategies = [ParallelStrategy.parse(s) for s in specs]
    uniq = list(dict.fromkeys(strategies))
    assert strategies[0].world_size <= world

    create_all_groups(uniq)  # collectively, on every rank, before any state is built
    ts = TrainingState(strategies[0]) if rank < strategies[0].world_size else None
    if ts is not None:
        ts.init_weights(a.seed)
    mgr = ElasticMegatronManager(uniq, training_state=ts, engine=a.engine)
    args = get_args()
    it = mgr.build_iterators(args.consumed_train_samples)[0]
    k = 0
    for iteration in range(1, a.train_iters + 1):
        if iteration > 1 and (iteration - 1) % a.switch_every == 0:
            # every rank meets here, active or idle (reference: check_reshard + global_barrier_by_gloo)
            mgr.global_barrier_by_gloo()
            k = (k + 1) % len(strategies)
            if strategies[k] != mgr.current:
                ckpt = dict(save_ckpt=True, ckpt_dir=os.path.join(a.save or "ckpt", f"reshard_{iteration}"))\
                    if a.save_around_reshard else {}
                ts = mgr.reshard(strategies[k], **ckpt)
                it = mgr.build_iterators(args.consumed_train_samples)[0] if ts is not None else None
                if ts is not None:
                    # the new layout's step hooks (the reference's loop re-binds its model config here)
                    ts.refresh_config(ts.model, ts.optimizer)
        if ts is None:
            args.consumed_train_samples += a.global_batch_size
            args.iteration = iteration
            continue
        t0 = time.perf_counter()
        out = train_step(ts, it)
        ms = (time.perf_counter() - t0) * 1e3
        args.consumed_train_samples += a.global_batch_size
        args.iteration = iteration
        if rank == 0:
            lr = ts.opt_param_scheduler.get_lr() if hasattr(ts.opt_param_scheduler, "get_lr") else float("nan")
            print(f" iteration {iteration:8d}/{a.train_iters:8d} | consumed samples: {args.consumed_train_samples:10d}"
                  f" | elapsed time per iteration (ms): {ms:.1f} | learning rate: {lr:.6E}"
                  f" | global batch size: {a.global_batch_size:5d} | lm loss: {out['loss']:.6E}"
                  f" | grad norm: {float(out['grad_norm']):.3f} | strategy: {mgr.current}", flush=True)
            tokens = a.global_batch_size * cfg.seq_length
            log_json("iteration", None, iteration=iteration, loss=out["loss"], ms=ms,
                     tokens_per_s_per_gpu=tokens / (ms / 1e3) / mgr.current.world_size, strategy=str(mgr.current))
    if a.save and ts is not None:
        from elasticmegatron_b200.runtime.checkpoint import save_checkpoint

        save_checkpoint(ts, a.save)
    mgr.global_barrier_by_gloo()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
