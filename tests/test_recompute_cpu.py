"""Full activation recompute (``TrainConfig(recompute=True)``): the same losses as storing activations under
every kind of parallelism whose forward holds collectives (TP + SP, PP 1F1B, EP all-to-all, CP), across a
switch, while keeping fewer tensors for backward."""
import numpy as np
import torch

from dist_utils import run_distributed


def _cfg(moe):
    from elasticmegatron_b200.config import ModelConfig

    return ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, num_query_groups=2, ffn_hidden_size=128,
                       vocab_size=500, seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2,
                       make_vocab_size_divisible_by=8, num_experts=4 if moe else None,
                       moe_ffn_hidden_size=64 if moe else None)


def _run(rank, world, specs, recompute, moe):
    from elasticmegatron_b200.config import Args, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    set_args(Args(model=_cfg(moe), train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3,
                                                     recompute=recompute, cp_comm_type="p2p")))
    S = [ParallelStrategy.parse(x) for x in dict.fromkeys(specs)]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(S, training_state=ts, engine="torch")
    consumed, losses = 0, []
    it = mgr.build_iterators(consumed)[0]
    for i, spec in enumerate(specs):
        if i and spec != specs[i - 1]:
            ts = mgr.reshard(spec)
            it = mgr.build_iterators(consumed)[0]
        losses.append(train_step(ts, it)["loss"])
        consumed += 8
    return losses


def test_recompute_keeps_the_losses():
    cases = [(2, ["ws2", "ws2"], False), (2, ["ws2-tp2", "ws2-tp2"], False), (2, ["ws2-pp2", "ws2-pp2"], False),
             (2, ["ws2-cp2", "ws2-cp2"], False), (2, ["ws2-ep2-etp1", "ws2-ep2-etp1"], True),
             (2, ["ws2", "ws2-tp2", "ws2-pp2"], False)]
    for world, specs, moe in cases:
        base = run_distributed(_run, world, specs, False, moe)[0]
        rec = run_distributed(_run, world, specs, True, moe)[0]
        np.testing.assert_allclose(rec, base, rtol=1e-6, err_msg=str(specs))


def test_recompute_saves_fewer_tensors():
    """One rank: count the elements kept for backward through the stage, with and without recompute (saved
    tensors plus, with recompute, the layer inputs the checkpoints hold)."""
    from elasticmegatron_b200.config import Args, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.training_state import TrainingState

    kept = {}
    for recompute in (False, True):
        set_args(Args(model=_cfg(False), train=TrainConfig(micro_batch_size=2, global_batch_size=2,
                                                           recompute=recompute)))
        ts = TrainingState(ParallelStrategy.parse("ws1"))
        ts.init_weights(0)
        ids = torch.randint(0, 500, (2, 32))
        n = [0]

        def pack(t):
            n[0] += t.numel()
            return t

        with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
            losses, _ = ts.stage(ids, ids)
        losses.sum().backward()
        # checkpointing holds each layer's input outside the hooks: count those too
        kept[recompute] = n[0] + (ts.stage.num_local_layers * 32 * 2 * 64 if recompute else 0)
    assert kept[True] < 0.5 * kept[False], kept
