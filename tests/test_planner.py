"""Reshard planner: every destination element is produced exactly from the right source element.

The oracle scatters one set of global tensors into the source and destination layouts independently
(``planner/materialize.py``); applying the plan to the source state must reproduce the destination state
bit for bit, including the SwiGLU halves, GQA group order, vocab padding and expert homes.
"""
import itertools

import numpy as np
import pytest
import torch

from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
from elasticmegatron_b200.parallel.strategy import ParallelStrategy
from elasticmegatron_b200.planner.layout import rank_layout
from elasticmegatron_b200.planner.materialize import init_global_params, scatter_to_rank
from elasticmegatron_b200.planner.plan import apply_plan_reference, build_plan, KIND_OPT

NAN = 12345.0


def _cfg(moe=False, tied=False):
    return ModelConfig(num_layers=4, hidden_size=64, num_attention_heads=8, num_query_groups=4, ffn_hidden_size=96,
                       vocab_size=300, params_dtype="fp32", max_tensor_parallel_size=4, make_vocab_size_divisible_by=8,
                       num_experts=8 if moe else None, moe_ffn_hidden_size=48 if moe else None,
                       untie_embeddings_and_output_weights=not tied)


def _state(cfg, s, g, og, overlap, bucket):
    P, O = {}, {}
    for r in range(s.world_size):
        rl = rank_layout(cfg, s, r, overlap, bucket)
        P[r] = torch.full((rl.param_numel,), float("nan"))
        O[r] = torch.full((3, rl.opt_numel), float("nan"))
        scatter_to_rank(cfg, s, r, g, P[r], O[r], og, overlap, bucket)
    return P, O


def _check_pair(cfg, a, b, overlap, bucket):
    g = init_global_params(cfg)
    gen = torch.Generator().manual_seed(1)
    og = {k: torch.stack([v, torch.rand(v.shape, generator=gen), torch.rand(v.shape, generator=gen)])
          for k, v in g.items()}
    plan = build_plan(a, b, cfg, overlap_grad_reduce=overlap, ddp_bucket_size=bucket)
    sP, sO = _state(cfg, a, g, og, overlap, bucket)
    dP, dO = _state(cfg, b, g, og, overlap, bucket)
    tP = {r: torch.full_like(v, float("nan")) for r, v in dP.items()}
    tO = {r: torch.full_like(v, float("nan")) for r, v in dO.items()}
    apply_plan_reference(plan, sO, sP, tO, tP)
    for r in dP:
        assert torch.equal(torch.nan_to_num(dP[r], NAN), torch.nan_to_num(tP[r], NAN)), (a, b, r)
        assert torch.equal(torch.nan_to_num(dO[r], NAN), torch.nan_to_num(tO[r], NAN)), (a, b, r)
    return plan


def _dense_strategies():
    out = []
    for tp in (1, 2, 4):
        for pp in (1, 2, 4):
            if 8 % (tp * pp) == 0:
                out.append(ParallelStrategy(world_size=8, tensor_model_parallel_size=tp,
                                            pipeline_model_parallel_size=pp))
    out.append(ParallelStrategy(world_size=4, tensor_model_parallel_size=2, pipeline_model_parallel_size=1))
    out.append(ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                                context_parallel_size=2))
    out.append(ParallelStrategy(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=2))
    return out


@pytest.mark.parametrize("overlap,bucket", [(False, None), (True, 3000)])
def test_all_dense_pairs(overlap, bucket):
    cfg = _cfg()
    set_args(Args(model=cfg, train=TrainConfig()))
    strats = _dense_strategies()
    for a, b in itertools.permutations(strats, 2):
        _check_pair(cfg, a, b, overlap, bucket)


def test_tied_embedding_pairs():
    """A tied word embedding is held by the first stage and, as the output layer, by the last: every switch
    writes both copies (including PP1 <-> PP>1, where the copy appears / disappears)."""
    from elasticmegatron_b200.planner.layout import rank_layout

    cfg = _cfg(tied=True)
    set_args(Args(model=cfg, train=TrainConfig()))
    strats = _dense_strategies()
    for a, b in itertools.permutations(strats, 2):
        _check_pair(cfg, a, b, True, 3000)
    pp2 = ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=2)
    names = {r: [lp.name for lp in rank_layout(cfg, pp2, r).params] for r in range(8)}
    first, last = pp2.coords(0)["pp"], pp2.coords(7)["pp"]
    assert first == 0 and last == 1
    assert "embedding.word_embeddings.weight" in names[0] and "output_layer.weight" not in names[0]
    assert names[7][-1] == "output_layer.weight" and "embedding.word_embeddings.weight" not in names[7]
    pp1 = ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=1)
    assert "output_layer.weight" not in [lp.name for lp in rank_layout(cfg, pp1, 0).params]


def test_moe_ep_pairs():
    cfg = _cfg(moe=True)
    set_args(Args(model=cfg, train=TrainConfig()))
    S = [ParallelStrategy(world_size=8, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                          expert_model_parallel_size=8, expert_tensor_parallel_size=1),
         ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=1,
                          expert_model_parallel_size=4, expert_tensor_parallel_size=1),
         ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=2,
                          expert_model_parallel_size=2, expert_tensor_parallel_size=1),
         ParallelStrategy(world_size=4, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                          expert_model_parallel_size=4, expert_tensor_parallel_size=1)]
    for a, b in itertools.permutations(S, 2):
        _check_pair(cfg, a, b, True, 5000)


def test_group_zero_replicas():
    cfg = _cfg()
    set_args(Args(model=cfg, train=TrainConfig()))
    a = ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=1,
                         num_distributed_optimizer_instances=2)
    b = ParallelStrategy(world_size=4, tensor_model_parallel_size=2, pipeline_model_parallel_size=1)
    down = _check_pair(cfg, a, b, False, None)
    # scale-down keeps the surviving instance's shards in place: all optimizer copies are local
    opt = down.desc[down.desc["kind"] == KIND_OPT]
    assert (opt["src_rank"] == opt["dst_rank"]).all()
    up = _check_pair(cfg, b, a, False, None)
    opt = up.desc[up.desc["kind"] == KIND_OPT]
    assert set(np.unique(opt["src_rank"]).tolist()) <= {0, 1, 2, 3}


def test_identity_plan_is_local_and_roofline_zero():
    cfg = _cfg()
    set_args(Args(model=cfg, train=TrainConfig()))
    a = ParallelStrategy(world_size=8, tensor_model_parallel_size=2, pipeline_model_parallel_size=2)
    p = build_plan(a, a, cfg, overlap_grad_reduce=False)
    assert (p.desc["src_rank"] == p.desc["dst_rank"]).all()
    assert p.nvlink_roofline_ms(770.0) == 0.0


def test_plan_describe_lists_every_parameter():
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.layout import virtual_params
    from elasticmegatron_b200.planner.plan import build_plan

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=100,
                      params_dtype="fp32", make_vocab_size_divisible_by=8, max_tensor_parallel_size=2)
    set_args(Args(model=cfg, train=TrainConfig()))
    a = ParallelStrategy(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)
    b = ParallelStrategy(world_size=2, tensor_model_parallel_size=2, pipeline_model_parallel_size=1)
    text = build_plan(a, b, cfg).describe(cfg)
    assert text.startswith("reshard plan ")
    for vp in virtual_params(cfg):
        assert vp.name in text
    assert "fp32 master+moments" in text and "->" in text
    short = build_plan(a, b, cfg).describe(cfg, ranks=[1], max_params=2)
    assert "more parameters" in short
