"""Tied word embedding / output layer (``untie_embeddings_and_output_weights=False``) on gloo ranks.

At PP=1 the head reads the embedding itself; at PP>1 the last stage holds a copy (``output_layer.weight``)
whose gradient is summed with the first stage's over the embedding group, so both copies take identical
steps.  The loss must not depend on the layout, switches must carry both copies, and the copies must stay
bitwise equal."""
import numpy as np

from dist_utils import run_distributed


def _run(rank, world, specs):
    import torch
    import torch.distributed as dist

    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, num_query_groups=2, ffn_hidden_size=128,
                      vocab_size=500, seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2,
                      make_vocab_size_divisible_by=8, untie_embeddings_and_output_weights=False)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3,
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
    # under PP>1: the first stage's embedding and the last stage's copy are bitwise equal (params and the
    # fp32 master / Adam moments, compared through the full local tensors)
    same = None
    if ts.ps.pp_size > 1:
        p = ts.stage.params_by_name
        mine = (p["embedding.word_embeddings.weight"] if ts.ps.is_first_stage else p["output_layer.weight"]).detach()
        other = torch.empty_like(mine)
        peer = ts.ps.group_ranks["embedding"]
        peer = [r for r in peer if r != rank][0]
        ops = [dist.P2POp(dist.isend, mine.contiguous(), peer), dist.P2POp(dist.irecv, other, peer)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()
        same = bool(torch.equal(mine, other))
    return losses, same


def test_tied_losses_do_not_depend_on_layout():
    base = run_distributed(_run, 2, ["ws2"] * 4)[0][0]
    for specs in (["ws2-tp2"] * 4, ["ws2-pp2"] * 4, ["ws2", "ws2-pp2", "ws2-tp2", "ws2-pp2"]):
        res = run_distributed(_run, 2, specs)
        np.testing.assert_allclose(res[0][0], base, rtol=1e-5, err_msg=str(specs))
        for losses, same in res:
            assert same in (None, True), specs


def test_tied_pp4_copies_stay_equal():
    res = run_distributed(_run, 4, ["ws4-pp2", "ws4-pp2", "ws4-tp2-pp2", "ws4-tp2-pp2"])
    base = run_distributed(_run, 4, ["ws4"] * 4)[0][0]
    np.testing.assert_allclose(res[0][0], base, rtol=1e-5)
    assert all(same is True for _, same in res)


def _ckpt(rank, world, root):
    import torch

    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.checkpoint import load_checkpoint, save_checkpoint
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, num_query_groups=2, ffn_hidden_size=128,
                      vocab_size=500, seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2,
                      make_vocab_size_divisible_by=8, untie_embeddings_and_output_weights=False)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    specs = ["ws2-pp2", "ws2", "ws2-tp2"]
    S = [ParallelStrategy.parse(x) for x in specs]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(S, training_state=ts, engine="torch")
    it = mgr.build_iterators(0)[0]
    train_step(ts, it)
    train_step(ts, it)
    save_checkpoint(ts, root, iteration=2, consumed_samples=16)
    ok = True
    for s in S[1:]:
        live = mgr.reshard(s)
        fresh = TrainingState(s)
        load_checkpoint(fresh, root)
        ok &= torch.equal(live.param_flat, fresh.param_flat) and torch.equal(live.opt_flat, fresh.opt_flat)
    return bool(ok)


def test_tied_checkpoint_pp2_loads_under_pp1_and_tp2(tmp_path):
    import torch

    assert all(run_distributed(_ckpt, 2, str(tmp_path)))
    it = tmp_path / "iter_0000002"
    first = torch.load(it / "mp_rank_00_000" / "model_optim_rng.pt", weights_only=False)["model"]
    last = torch.load(it / "mp_rank_00_001" / "model_optim_rng.pt", weights_only=False)["model"]
    # Megatron's naming: the last stage saves its copy of the tied embedding as the output layer
    assert "embedding.word_embeddings.weight" in first and "output_layer.weight" not in first
    assert "output_layer.weight" in last and "embedding.word_embeddings.weight" not in last
    assert torch.equal(first["embedding.word_embeddings.weight"], last["output_layer.weight"])
