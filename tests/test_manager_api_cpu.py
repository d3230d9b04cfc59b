"""The reference-API entry points of the manager and the training state on gloo ranks, each checked by its
effect: ``register`` (a custom state builder and dataset provider are the ones used), ``get_data_parallel_group``,
``global_barrier_by_gloo``, meta-device switches (they leave the live state untouched) followed by
``clear_meta_state``, ``release`` / ``rebuild`` (arenas return to the pool and come back),
``update_model_weight`` (parameters regenerated from the fp32 master and all-gathered over DP) and
``refresh_config``."""
from dist_utils import run_distributed


def _api(rank, world):
    import torch
    import torch.distributed as dist

    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import MockGPTDataset
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                      seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    out = {}
    built = []

    def setup(strategy, is_meta_device=False):
        built.append((str(strategy), is_meta_device))
        return TrainingState(strategy, is_meta_device=is_meta_device)

    provided = []

    def provider():
        provided.append(1)
        return MockGPTDataset(1 << 20, cfg.seq_length, cfg.vocab_size, seed=99), None, None

    ElasticMegatronManager.register(setup, provider)
    specs = ["ws2", "ws2-tp2", "ws1"]
    S = [ParallelStrategy.parse(s) for s in specs]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(specs, training_state=ts, engine="torch")

    # data comes from the registered provider
    ids, _ = next(iter(mgr.build_iterators(0)[0]))
    want = MockGPTDataset(1 << 20, cfg.seq_length, cfg.vocab_size, seed=99)[rank * 2][:-1]
    out["provider"] = bool(provided) and torch.equal(ids[0], want)

    # groups and the host barrier
    g = mgr.get_data_parallel_group("ws2")
    out["dp_group"] = g is not None and dist.get_world_size(g) == 2
    g1 = mgr.get_data_parallel_group("ws1")
    out["dp_idle"] = (g1 is None) if rank == 1 else True
    mgr.global_barrier_by_gloo()

    train_step(ts, mgr.build_iterators(0)[0])
    # meta-device switches there and back: the registered builder makes a meta state, no data moves and the
    # live state is neither released nor changed
    before_p, before_o = ts.param_flat.clone(), ts.opt_flat.clone()
    mgr.reshard("ws2-tp2", is_meta_device=True)
    out["meta_built"] = ("ws2-tp2-pp1-cp1-dp1-ep1-etp2-inst1-sp", True) in built
    back = mgr.reshard("ws2", is_meta_device=True)
    out["live_kept"] = (back is ts and not ts.model_released and torch.equal(ts.param_flat, before_p)
                        and torch.equal(ts.opt_flat, before_o))
    mgr.clear_meta_state("ws2-tp2")
    # a real switch and back: the registered builder builds the cleared state again, for real
    tp = mgr.reshard("ws2-tp2")
    out["real_built"] = ("ws2-tp2-pp1-cp1-dp1-ep1-etp2-inst1-sp", False) in built and not tp.is_meta_device
    back = mgr.reshard("ws2")
    out["round_trip"] = torch.equal(back.param_flat, before_p) and torch.equal(back.opt_flat, before_o)

    # release returns the arenas to the pool; rebuild takes arenas back (contents are refilled by a switch)
    tp.release()
    out["released"] = tp.model_released and tp.optimizer_released and tp.param_arena is None
    tp.rebuild()
    out["rebuilt"] = (not tp.model_released) and tp.param_flat.numel() == tp.layout.param_numel
    tp.release()

    # update_model_weight: parameters regenerated from the fp32 master of each shard, then all-gathered
    good = back.param_flat.clone()
    back.param_flat.zero_()
    back.update_model_weight()
    out["update_model_weight"] = torch.equal(back.param_flat, good)
    hooks = back.refresh_config(back.model, back.optimizer)
    ok = all(getattr(c, "step_hooks", None) is hooks for c in back.model) and hooks.ddp is back.ddp
    with hooks.no_sync_func():
        ok &= back.ddp.sync_enabled is False
    ok &= back.ddp.sync_enabled is True and hooks.grad_scale_func(3.0) == 3.0
    try:
        back.refresh_config(back.model, object())  # an optimizer of another layout
        ok = False
    except ValueError:
        pass
    out["refresh_config"] = bool(ok)
    # the reference's constructor form: the live model (and its optimizer / scheduler) instead of the state
    m2 = ElasticMegatronManager(specs, model=back.model, optimizer=back.optimizer,
                                opt_param_scheduler=back.opt_param_scheduler, engine="torch")
    out["model_ctor"] = m2.training_state is back
    ElasticMegatronManager.register(None, None)
    return out


def test_reference_api_entry_points():
    for res in run_distributed(_api, 2):
        assert all(res.values()), res


def _ckpt_and_logger(rank, world, root):
    import json
    import logging

    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, get_args, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                      seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    S = [ParallelStrategy.parse(s) for s in ("ws2", "ws2-tp2")]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(S, training_state=ts, engine="torch")
    train_step(ts, mgr.build_iterators(0)[0])
    get_args().iteration = 1

    records = []

    class _Keep(logging.Handler):
        def emit(self, rec):
            records.append(rec.getMessage())

    log = logging.getLogger(f"switch-test-{rank}")
    log.addHandler(_Keep())
    log.setLevel(logging.INFO)
    log.propagate = False
    mgr.reshard("ws2-tp2", logger=log, save_ckpt=True, ckpt_dir=root)
    rec = [json.loads(m) for m in records if m.startswith("{")]
    return len(rec) == 1 and rec[0]["event"] == "reshard" and rec[0]["dst"].startswith("ws2-tp2")


def test_reshard_saves_both_sides_and_logs_to_the_logger(tmp_path):
    """``reshard(save_ckpt=True, ckpt_dir=...)`` writes the source layout to before_reshard/ and the destination
    to after_reshard/; converting the first offline to the destination layout gives the second exactly (the
    reference's convert-and-compare check).  The switch record goes to the given logger on every rank."""
    import os

    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.checkpoint import convert_checkpoint
    from elasticmegatron_b200.tools.compare_ckpt import compare

    assert all(run_distributed(_ckpt_and_logger, 2, str(tmp_path)))
    before, after = tmp_path / "before_reshard", tmp_path / "after_reshard"
    ib = next(d for d in os.listdir(before) if d.startswith("iter_"))
    ia = next(d for d in os.listdir(after) if d.startswith("iter_"))
    assert sorted(os.listdir(before / ib)) == ["mp_rank_00"]
    assert sorted(os.listdir(after / ia)) == ["mp_rank_00", "mp_rank_01"]
    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                      seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    conv = tmp_path / "converted"
    convert_checkpoint(str(before), str(conv), ParallelStrategy.parse("ws2-tp2"))
    ic = next(d for d in os.listdir(conv) if d.startswith("iter_"))
    assert compare(str(conv / ic), str(after / ia), 0.0) == []
    # the same check through the command line the README gives
    from elasticmegatron_b200.tools import convert_ckpt

    assert convert_ckpt.main([str(before), str(tmp_path / "cli"), "--world-size", "2", "--tp", "2",
                              "--compare", str(after)]) == 0


def _sp_switch(rank, world, specs):
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.manager import ElasticMegatronManager
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                      seq_length=32, params_dtype="fp32", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    S = [ParallelStrategy.parse(s) for s in dict.fromkeys(specs)]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    mgr = ElasticMegatronManager(S, training_state=ts, engine="torch")
    ptr, allocated = ts.param_flat.data_ptr(), ts.pool.allocated_bytes
    losses, moved, same_arenas = [], [], True
    for i, s in enumerate(specs):
        if i and s != specs[i - 1]:
            ts = mgr.reshard(s)
            moved.append(mgr.last_switch["gbytes"])
            same_arenas &= ts.param_flat.data_ptr() == ptr and ts.pool.allocated_bytes == allocated
        losses.append(train_step(ts, mgr.build_iterators(8 * i)[0])["loss"])
    return losses, moved, same_arenas


def test_sp_only_switch_hands_over_the_arenas():
    """Strategies that differ only in sequence parallelism share a layout: a switch between them hands the
    arenas over (no copy, no allocation) and training continues as if nothing happened."""
    import numpy as np

    base = run_distributed(_sp_switch, 2, ["ws2-tp2"] * 4)
    sw = run_distributed(_sp_switch, 2, ["ws2-tp2", "ws2-tp2-nosp", "ws2-tp2-nosp", "ws2-tp2"])
    np.testing.assert_allclose(sw[0][0], base[0][0], rtol=1e-5)
    for losses, moved, same in sw:
        assert moved == [0.0, 0.0] and same, (moved, same)


def test_synthetic_dataset_follows_the_model_shape():
    """A second model in the same process (another sequence length / vocabulary) gets samples of its own shape,
    not the first model's cached ones; a registered dataset provider is still called once."""
    from elasticmegatron_b200.config import ModelConfig
    from elasticmegatron_b200.runtime.data import DataloaderState

    DataloaderState.register(None)
    a = ModelConfig(num_layers=1, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=1000,
                    seq_length=64)
    b = ModelConfig(num_layers=1, hidden_size=64, num_attention_heads=4, ffn_hidden_size=128, vocab_size=500,
                    seq_length=32)
    da = DataloaderState.get_datasets(a, 0)[0]
    db = DataloaderState.get_datasets(b, 0)[0]
    assert da is not db
    assert DataloaderState.get_datasets(b, 0)[0] is db
    calls = []
    DataloaderState.register(lambda: calls.append(1) or ("ds", None, None))
    assert DataloaderState.get_datasets(a, 0)[0] == "ds" and DataloaderState.get_datasets(b, 0)[0] == "ds"
    assert len(calls) == 1
    DataloaderState.register(None)
