"""Context parallelism on gloo ranks: a CP2 run equals a DP2 run of the same global batch, and a CP2 <-> DP2
switch keeps the loss curve."""
import numpy as np

from dist_utils import run_distributed

CP = [dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1),
      dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1, context_parallel_size=2)]


def _run(rank, world, schedule, gqa, cp_comm_type="all_gather"):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, num_query_groups=2 if gqa else 4,
                      ffn_hidden_size=128, vocab_size=500, seq_length=32, params_dtype="fp32",
                      max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3,
                                               cp_comm_type=cp_comm_type)))
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


def _ring_vs_gather(rank, world, gqa):
    import torch
    import torch.distributed as dist

    from elasticmegatron_b200.parallel.context_parallel import (cp_attention, cp_ring_attention,
                                                                cp_ulysses_attention)

    G, hpg, d, b, s = (4, 2, 16, 2, 12) if gqa else (4, 1, 16, 2, 12)
    gen = torch.Generator().manual_seed(7)
    # one global sequence; rank r holds global chunks r and 2*CP-1-r
    full = torch.randn(2 * world * (s // 2), b, G, hpg + 2, d, generator=gen, dtype=torch.float64)
    dfull = torch.randn(2 * world * (s // 2), b, G * hpg * d, generator=gen, dtype=torch.float64)
    c = s // 2
    idx = torch.cat([torch.arange(rank * c, (rank + 1) * c),
                     torch.arange((2 * world - 1 - rank) * c, (2 * world - rank) * c)])
    mine, dmine = full[idx].float(), dfull[idx].float()
    out = {}
    res = []
    for fn in (cp_attention, cp_ring_attention, cp_ulysses_attention):
        x = mine.clone().requires_grad_()
        y = fn(x, hpg, dist.group.WORLD, rank, world)
        y.backward(dmine)
        res.append((y.detach(), x.grad))
    out["fwd"] = max((res[0][0] - r[0]).abs().max().item() for r in res[1:])
    out["bwd"] = max((res[0][1] - r[1]).abs().max().item() for r in res[1:])
    # the whole-sequence oracle on every rank: plain causal attention of the global sequence (fp64), and its
    # gradient for the loss sum over ranks of <out_r, dout_r> = <out, dfull>
    F = full.clone().requires_grad_()
    q = F[:, :, :, :hpg].permute(1, 2, 3, 0, 4)
    k, v = F[:, :, :, hpg].permute(1, 2, 0, 3), F[:, :, :, hpg + 1].permute(1, 2, 0, 3)
    sc = torch.einsum("bghid,bgjd->bghij", q, k) / d ** 0.5
    n = sc.shape[-1]
    sc = sc.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    o = torch.einsum("bghij,bgjd->bghid", sc.softmax(-1), v).permute(3, 0, 1, 2, 4).reshape(n, b, -1)
    (o * dfull).sum().backward()
    out["oracle"] = max((o[idx].detach().float() - r[0]).abs().max().item() for r in res)
    out["oracle_bwd"] = max((F.grad[idx].float() - r[1]).abs().max().item() for r in res)
    return out


def test_ring_and_ulysses_attention_match_all_gather():
    """cp_comm_type p2p (ring) and a2a (Ulysses) against all_gather, and all three against causal attention
    of the unsplit sequence (forward and gradients)."""
    for world in (2, 4):
        for gqa in (False, True):
            for r in run_distributed(_ring_vs_gather, world, gqa):
                assert max(r.values()) < 1e-5, (world, gqa, r)


def test_cp2_ring_and_ulysses_equal_dp2():
    dp = run_distributed(_run, 2, [0, 0, 0], True)[0]
    for kind in ("p2p", "a2a"):
        cp = run_distributed(_run, 2, [1, 1, 1], True, kind)[0]
        np.testing.assert_allclose(dp, cp, rtol=1e-5, err_msg=kind)
