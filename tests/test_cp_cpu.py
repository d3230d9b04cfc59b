"""Context parallelism on gloo ranks: a CP2 run equals a DP2 run of the same global batch, and a CP2 <-> DP2
switch keeps the loss curve."""
import numpy as np

from dist_utils import run_distributed

CP = [dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1),
      dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1, context_parallel_size=2)]


def _run(rank, world, schedule, gqa):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, num_query_groups=2 if gqa else 4,
                      ffn_hidden_size=128, vocab_size=500, seq_length=32, params_dtype="fp32",
                      max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    S = [ParallelStrategy(**s) for s in CP]
    create_all_groups(S)
    ts = TrainingState(S[schedule[0]])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(CP, training_state=ts, engine="torch") if schedule[0] == 0 else None
    if mgr is None:
        mgr = ElasticMegatronManager([CP[1], CP[0]], training_state=ts, engine="torch")
    consumed, losses = 0, []
    it = mgr.build_iterators(consumed)[0]
    for i, k in enumerate(schedule):
        if i and k != schedule[i - 1]:
            ts = mgr.reshard(CP[k])
            it = mgr.build_iterators(consumed)[0]
        losses.append(train_step(ts, it)["loss"])
        consumed += 8
    return losses


def test_cp2_equals_dp2_and_switch_keeps_loss():
    for gqa in (False, True):
        dp = run_distributed(_run, 2, [0, 0, 0, 0], gqa)[0]
        cp = run_distributed(_run, 2, [1, 1, 1, 1], gqa)[0]
        sw = run_distributed(_run, 2, [0, 1, 1, 0], gqa)[0]
        np.testing.assert_allclose(dp, cp, rtol=1e-5)
        np.testing.assert_allclose(dp, sw, rtol=1e-5)


CP4 = [dict(world_size=4, tensor_model_parallel_size=2, pipeline_model_parallel_size=1),
       dict(world_size=4, tensor_model_parallel_size=2, pipeline_model_parallel_size=1, context_parallel_size=2),
       dict(world_size=4, tensor_model_parallel_size=1, pipeline_model_parallel_size=2, context_parallel_size=2)]


def _run4(rank, world, schedule):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, num_query_groups=2, ffn_hidden_size=128,
                      vocab_size=500, seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2,
                      make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    S = [ParallelStrategy(**s) for s in CP4]
    create_all_groups(S)
    ts = TrainingState(S[schedule[0]])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(CP4, training_state=ts, engine="torch")
    consumed, losses = 0, []
    it = mgr.build_iterators(consumed)[0]
    for i, k in enumerate(schedule):
        if i and k != schedule[i - 1]:
            ts = mgr.reshard(CP4[k])
            it = mgr.build_iterators(consumed)[0]
        losses.append(train_step(ts, it)["loss"])
        consumed += 8
    return losses


def test_cp_combined_with_tp_and_pp_switches():
    """TP2*DP2 -> TP2*CP2 (SP + CP) -> PP2*CP2 -> TP2*DP2 on 4 ranks keeps the loss of the no-switch run."""
    base = run_distributed(_run4, 4, [0, 0, 0, 0])[0]
    sw = run_distributed(_run4, 4, [0, 1, 2, 0])[0]
    np.testing.assert_allclose(base, sw, rtol=1e-5)
