"""The switching phases of bench.py (tokens/s per strategy of BASELINE config 2's schedule, switch latency per
consecutive pair with state checksums, the other engines on the first pair) run end to end on 4 and 8 gloo ranks
with a small model, so every rank takes the same collectives in the same order at the GPU counts the scaling
run uses; every switch must keep the layout-independent checksum of the whole state."""
import pytest

from dist_utils import run_distributed


def _phases(rank, world):
    import argparse
    import time

    import torch
    import torch.distributed as dist

    import bench
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=128, num_attention_heads=8, ffn_hidden_size=256, vocab_size=512,
                      seq_length=64, params_dtype="fp32", max_tensor_parallel_size=8, make_vocab_size_divisible_by=8)
    gbs = 2 * world
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=1, global_batch_size=gbs, lr=1e-3,
                                               overlap_grad_reduce=True, overlap_param_gather=True, seed=0)))
    sched = bench.schedule_for(world)
    base = dict(world_size=world, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                sequence_parallel=False)
    S = ParallelStrategy(**base)
    strategies = [base] + [s for s in sched if ParallelStrategy(**s) != S]
    create_all_groups([ParallelStrategy(**s) for s in strategies])
    ts = TrainingState(S)
    ts.init_weights(0)

    def barrier():
        dist.barrier()

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def timed_steps(state, itr, n):
        barrier()
        t0 = time.perf_counter()
        for _ in range(n):
            train_step(state, itr, return_loss=False)
        barrier()
        return (time.perf_counter() - t0) * 1e3

    args = argparse.Namespace(strategy_steps=1, reshard_iters=1, no_context=False)
    per, switches, context, link, ok = bench.switching_phases(args, world, strategies, sched, ts, gbs * cfg.seq_length,
                                                              timed_steps, barrier, max_over_ranks)
    return ([p["strategy"] for p in per], [p["tokens_per_s"] > 0 for p in per],
            [(w["src"], w["dst"], w["checksum_ok"]) for w in switches], sorted(k for k in context if k != "note"), ok)


@pytest.mark.parametrize("world", [4, 8])
def test_bench_switching_phases_on_host_ranks(world):
    import bench

    res = run_distributed(_phases, world, timeout=900.0)
    names, positive, switches, engines, ok = res[0]
    assert all(r == res[0] for r in res)  # every rank reports the same schedule
    assert len(names) == len(bench.schedule_for(world)) and all(positive)
    assert ok and all(c for _, _, c in switches) and len(switches) == len(names)
    assert engines == ["reference", "torch"]
