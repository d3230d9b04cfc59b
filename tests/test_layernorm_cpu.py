"""Megatron's LayerNorm (``normalization="LayerNorm"``, a weight and a bias per norm; the reference demo's
model) on gloo ranks: the biases are part of every layout, train, and the loss does not depend on the layout
or on switches."""
import itertools

import numpy as np

from dist_utils import run_distributed


def _cfg():
    from elasticmegatron_b200.config import ModelConfig

    return ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                       seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8,
                       normalization="LayerNorm")


def _run(rank, world, specs):
    import torch

    from elasticmegatron_b200.config import Args, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    set_args(Args(model=_cfg(), train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3,
                                                  overlap_grad_reduce=True, ddp_bucket_size=20000)))
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
    biases = [p for n, p in ts.stage.params_by_name.items() if n.endswith("bias")]
    trained = bool(biases) and all(float(p.detach().abs().max()) > 0 for p in biases)
    return losses, trained


def test_layernorm_losses_do_not_depend_on_layout():
    base = run_distributed(_run, 2, ["ws2"] * 4)
    assert all(t for _, t in base)  # every bias left zero after training
    for specs in (["ws2-tp2"] * 4, ["ws2-tp2-nosp"] * 4, ["ws2-pp2"] * 4, ["ws2", "ws2-tp2", "ws2-pp2", "ws2"]):
        res = run_distributed(_run, 2, specs)
        np.testing.assert_allclose(res[0][0], base[0][0], rtol=1e-5, err_msg=str(specs))
        assert all(t for _, t in res), specs


def test_layernorm_planner_pairs_and_demo_preset():
    import torch

    from elasticmegatron_b200.config import Args, TrainConfig, preset, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.layout import rank_layout, virtual_params
    from test_planner import _check_pair

    cfg = _cfg()
    cfg.num_layers, cfg.max_tensor_parallel_size = 4, 4
    set_args(Args(model=cfg, train=TrainConfig()))
    S = [ParallelStrategy.parse(s) for s in ("ws8", "ws8-tp2", "ws8-tp4-pp2", "ws4-pp4", "ws8-cp2")]
    for a, b in itertools.permutations(S, 2):
        _check_pair(cfg, a, b, True, 3000)
    names = [vp.name for vp in virtual_params(cfg)]
    assert "decoder.layers.0.self_attention.linear_qkv.layer_norm_bias" in names
    assert "decoder.layers.0.mlp.linear_fc1.layer_norm_bias" in names and "decoder.final_layernorm.bias" in names
    assert sum(torch.Size(vp.shape).numel() for vp in virtual_params(cfg)) == cfg.num_params()
    demo = preset("demo-tiny")
    assert demo.normalization == "LayerNorm" and demo.num_layers == 4 and demo.hidden_size == 4096
    set_args(Args(model=demo, train=TrainConfig()))
    rl = rank_layout(demo, ParallelStrategy.parse("ws8-tp2"), 0)
    assert any(lp.name.endswith("layer_norm_bias") for lp in rl.params)
