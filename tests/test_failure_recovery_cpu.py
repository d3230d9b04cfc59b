"""Failure detection and recovery on CPU/gloo ranks (no GPU is faulted; the failure is a rank that stops).

Four ranks train under DP4 with two Group-ZeRO optimizer instances (each optimizer shard has a replica on
another rank).  Rank 3 stops heartbeating and leaves between steps.  The survivors' watchdog reports it from
the store alone; ranks 0 and 1 then ``recover`` onto DP2, reading only surviving replicas and using only the
new strategy's groups, and the next loss equals that of an orderly reshard of the same schedule.
"""
import datetime
import os
import traceback

import numpy as np
import torch.multiprocessing as mp

from dist_utils import free_port

STRATS = [dict(world_size=4, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
               num_distributed_optimizer_instances=2),
          dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)]


def _body(rank, fail):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.health import Heartbeat, Watchdog
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                      seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    S = [ParallelStrategy(**s) for s in STRATS]
    create_all_groups(S)
    hb = Heartbeat(rank, interval=0.1).start()
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(STRATS, training_state=ts, engine="torch")
    it = mgr.build_iterators(0)[0]
    train_step(ts, it)
    train_step(ts, it)
    if not fail:
        ts = mgr.reshard(STRATS[1])
        if ts is None:
            return None
        return train_step(ts, mgr.build_iterators(16)[0])["loss"]
    if rank == 3:  # the failing rank leaves between steps: no kernel or collective in flight
        hb.stop()
        return "left"
    dead = Watchdog(range(4), timeout=1.0).wait_for_failure(limit=30)
    assert dead == {3}, dead
    ts = mgr.recover(STRATS[1], dead)
    if ts is None:
        return "idle"
    return train_step(ts, mgr.build_iterators(16)[0])["loss"]


def _entry(rank, world, port, fail, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        q.put((rank, "ok", _body(rank, fail)))
        if not fail:
            dist.barrier()
    except Exception:
        q.put((rank, "err", traceback.format_exc()))
    q.close()
    q.join_thread()  # flush the result before leaving
    os._exit(0)  # no teardown collective: a peer may be gone


def _run(fail):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_entry, args=(r, 4, port, fail, q)) for r in range(4)]
    for p in ps:
        p.start()
    res = dict((r, (st, v)) for r, st, v in (q.get(timeout=300) for _ in range(4)))
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    for r, (st, v) in res.items():
        assert st == "ok", v
    return {r: v for r, (st, v) in res.items()}


def test_detect_and_recover_from_lost_rank():
    ref = _run(False)
    got = _run(True)
    assert got[3] == "left" and got[2] == "idle"
    np.testing.assert_allclose([got[0], got[1]], [ref[0], ref[1]], rtol=1e-6)
