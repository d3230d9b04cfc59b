"""Group-ZeRO redundancy switches on 4 gloo ranks, and the failure detector on its own.

* DP4 with two optimizer instances -> DP2 (one instance, ranks 2-3 idle) -> DP4 with two instances again while
  training: the losses equal a run that never switches (the replica is dropped, then rebuilt from the
  surviving shards - the reference's ``redundant_backup``, elastic_manager.py:124-141, as a plan);
* heartbeat / watchdog against an in-process store: a rank that stops beating is reported once its last beat is
  older than the timeout, a rank that never beat is reported at once.
"""
import time

import numpy as np

from dist_utils import run_distributed

STRATS = [dict(world_size=4, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
               num_distributed_optimizer_instances=2),
          dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1),
          dict(world_size=4, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)]


def _run(rank, world, schedule):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                      seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    S = [ParallelStrategy(**s) for s in STRATS]
    create_all_groups(S)
    ts = TrainingState(S[schedule[0]])
    ts.init_weights(0)
    order = [STRATS[schedule[0]]] + [s for i, s in enumerate(STRATS) if i != schedule[0]]
    mgr = ElasticMegatronManager(order, training_state=ts, engine="torch")
    consumed, losses = 0, []
    it = mgr.build_iterators(consumed)[0]
    for i, k in enumerate(schedule):
        if i and k != schedule[i - 1]:
            ts = mgr.reshard(STRATS[k])
            it = mgr.build_iterators(consumed)[0] if ts is not None else None
        losses.append(train_step(ts, it)["loss"] if ts is not None else None)
        consumed += 8
    return losses


def test_instance_count_switch_keeps_the_loss():
    base = run_distributed(_run, 4, [0, 0, 0, 0, 0])[0]
    sw = run_distributed(_run, 4, [0, 1, 1, 0, 2])
    np.testing.assert_allclose(base, sw[0], rtol=2e-6)
    assert sw[2][1] is None and sw[3][2] is None  # ranks 2-3 idle while the world is 2


def test_heartbeat_watchdog():
    import torch.distributed as dist

    from elasticmegatron_b200.runtime.health import Heartbeat, Watchdog

    store = dist.HashStore()
    hb0 = Heartbeat(0, store=store, interval=0.05).start()
    hb1 = Heartbeat(1, store=store, interval=0.05).start()
    wd = Watchdog([0, 1, 2], store=store, timeout=0.5)
    assert wd.failed_ranks() == {2}  # never beat
    hb1.stop()
    time.sleep(0.8)
    assert wd.failed_ranks() == {1, 2}
    hb0.stop()
