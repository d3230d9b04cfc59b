"""K1 reshard copy kernel: byte-exact against the planner's CPU oracle.

``test_k1_emulated_ranks`` runs on one GPU: all ranks' arenas of both layouts live on the device and every
rank's task table is executed, once as in pull mode (tables of the destination ranks) and once as in push mode
(tables of the source ranks).  ``test_native_engine_two_gpus`` runs the real
engine (CUDA IPC + NCCL barriers) in two processes and needs two GPUs.
"""
import itertools

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args

    cfg = ModelConfig(num_layers=4, hidden_size=128, num_attention_heads=8, num_query_groups=4, ffn_hidden_size=192,
                      vocab_size=1000, params_dtype="bf16", max_tensor_parallel_size=4, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(overlap_grad_reduce=True, ddp_bucket_size=20000)))
    return cfg


def _state(cfg, s, g, og):
    from elasticmegatron_b200.planner.layout import rank_layout
    from elasticmegatron_b200.planner.materialize import scatter_to_rank

    P, O = {}, {}
    for r in range(s.world_size):
        rl = rank_layout(cfg, s, r, True, 20000)
        p = torch.zeros(rl.param_numel)
        o = torch.zeros(3, rl.opt_numel)
        scatter_to_rank(cfg, s, r, g, p, o, og, True, 20000)
        P[r], O[r] = p.bfloat16().cuda(), o.cuda()
    return P, O


def test_k1_emulated_ranks():
    from elasticmegatron_b200.ops.native import ext
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.planner.materialize import init_global_params
    from elasticmegatron_b200.planner.plan import build_plan
    from elasticmegatron_b200.transfer.native_engine import NativeP2PEngine

    cfg = _cfg()
    g = {k: v.bfloat16().float() for k, v in init_global_params(cfg).items()}
    og = {k: torch.stack([v, torch.rand_like(v), torch.rand_like(v)]) for k, v in g.items()}
    S = [ParallelStrategy(world_size=8, tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp)
         for tp, pp in ((1, 1), (2, 2), (4, 1), (1, 4))]
    S.append(ParallelStrategy(world_size=4, tensor_model_parallel_size=2, pipeline_model_parallel_size=1))
    for mode, (a, b) in itertools.product(("pull", "push"), itertools.permutations(S, 2)):
        eng = NativeP2PEngine(mode=mode, task_bytes=4096)  # small tasks: exercise the splitter
        plan = build_plan(a, b, cfg)
        sP, sO = _state(cfg, a, g, og)
        eP, eO = _state(cfg, b, g, og)
        tP = {r: torch.full_like(v, float("nan")) for r, v in eP.items()}
        tO = {r: torch.full_like(v, float("nan")) for r, v in eO.items()}
        addrs = {r: (sP[r].data_ptr() if r in sP else 0, sO[r].data_ptr() if r in sO else 0,
                     tP[r].data_ptr() if r in tP else 0, tO[r].data_ptr() if r in tO else 0)
                 for r in range(max(a.world_size, b.world_size))}
        for r in range(b.world_size if mode == "pull" else a.world_size):
            t = eng._tasks(plan, r, addrs, 2)
            if len(t):
                buf = torch.from_numpy(t.view(np.uint8).copy()).cuda()
                ext().reshard_copy(buf, len(t), 0)
        torch.cuda.synchronize()
        for r in range(b.world_size):
            # padding is never written by the plan: compare only what the oracle defines (non-nan after copy)
            mP, mO = ~torch.isnan(tP[r].float()), ~torch.isnan(tO[r])
            assert torch.equal(tP[r][mP], eP[r][mP]) and torch.equal(tO[r][mO], eO[r][mO]), (mode, a, b, r)
            # every non-padding element was written
            nzP = eP[r] != 0
            assert bool(mP[nzP].all()), (mode, a, b, r)


def _two_gpu(rank, world):
    import torch

    torch.cuda.set_device(rank)
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, ffn_hidden_size=512, vocab_size=1000,
                      seq_length=128, params_dtype="bf16", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4)))
    strats = [dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1),
              dict(world_size=2, tensor_model_parallel_size=2, pipeline_model_parallel_size=1),
              dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=2)]
    S = [ParallelStrategy(**s) for s in strats]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(strats, training_state=ts, engine="native")
    it = mgr.build_iterators(0)[0]
    train_step(ts, it)
    P0, O0 = ts.param_flat.clone(), ts.opt_flat.clone()
    for i in (1, 2, 0):
        ts = mgr.reshard(strats[i])
    ok = bool(torch.equal(P0, ts.param_flat) and torch.equal(O0, ts.opt_flat))
    return ok


def test_native_engine_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    assert all(run_distributed(_two_gpu, 2, backend="nccl"))


def _group_zero_two_gpus(rank, world):
    """Group-ZeRO on two GPUs with the native engine: DP2 with two optimizer instances (each GPU a full replica)
    -> one GPU (the replica dropped, rank 1 idle) -> DP2 with two instances again (the replica rebuilt by K1
    over NVLink from the surviving copy).  Every byte of the state must come back, on both GPUs."""
    import torch
    torch.cuda.set_device(rank)
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, ffn_hidden_size=512, vocab_size=1000,
                      seq_length=128, params_dtype="bf16", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4)))
    strats = [dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                   num_distributed_optimizer_instances=2),
              dict(world_size=1, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)]
    S = [ParallelStrategy(**s) for s in strats]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(strats, training_state=ts, engine="native")
    train_step(ts, mgr.build_iterators(0)[0])
    P0, O0 = ts.param_flat.clone(), ts.opt_flat.clone()
    mid = mgr.reshard(strats[1])
    ok = (mid is None) == (rank == 1)
    if mid is not None:
        ok &= torch.equal(mid.opt_flat, O0) and torch.equal(mid.param_flat, P0)
    back = mgr.reshard(strats[0])
    ok &= torch.equal(back.param_flat, P0) and torch.equal(back.opt_flat, O0)
    loss = train_step(back, mgr.build_iterators(4)[0])["loss"]
    return bool(ok), loss


def test_group_zero_replica_rebuild_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    res = run_distributed(_group_zero_two_gpus, 2, backend="nccl")
    assert all(r[0] for r in res), res
    assert res[0][1] == res[1][1]
