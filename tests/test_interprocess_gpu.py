"""Inter-process scale-down on two GPUs: a 2-rank NCCL job exports its arenas as CUDA IPC handles; a separate
1-rank process maps them and pulls its own layout from both GPUs' memory with the K1 kernel.  The adopted state
must equal, bit for bit, the same state loaded from a checkpoint under the new strategy."""
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

STRATS = [dict(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1),
          dict(world_size=1, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)]


def _setup():
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, ffn_hidden_size=512, vocab_size=1000,
                      seq_length=128, params_dtype="bf16", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4)))


def _old(rank, world, root):
    from elasticmegatron_b200.config import get_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.checkpoint import save_checkpoint
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.interprocess import export_state, wait_for_acks
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    _setup()
    S = [ParallelStrategy(**s) for s in STRATS]
    create_all_groups(S)
    ts = TrainingState(S[0])
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    train_step(ts, it)
    train_step(ts, it)
    torch.cuda.synchronize()
    get_args().iteration, get_args().consumed_train_samples = 2, 8
    save_checkpoint(ts, os.path.join(root, "ckpt"), iteration=2, consumed_samples=8)
    export_state(ts, root, "down")
    wait_for_acks(root, "down", 1, timeout=180)
    return True


def _new(root, q):
    try:
        torch.cuda.set_device(0)
        _setup()
        from elasticmegatron_b200.parallel.strategy import ParallelStrategy
        from elasticmegatron_b200.runtime.checkpoint import load_checkpoint
        from elasticmegatron_b200.runtime.interprocess import ack, adopt, import_records
        from elasticmegatron_b200.runtime.training_state import TrainingState

        s = ParallelStrategy(**STRATS[1])
        ts = TrainingState(s)
        recs = import_records(root, "down", old_world=2, timeout=180)
        adopt(ts, recs)
        ack(root, "down", 0)
        ref = TrainingState(s)
        load_checkpoint(ref, os.path.join(root, "ckpt"))
        ok = torch.equal(ts.param_flat, ref.param_flat) and torch.equal(ts.opt_flat, ref.opt_flat)
        q.put(("ok", bool(ok)))
    except Exception as e:  # pragma: no cover
        import traceback

        q.put(("err", traceback.format_exc()))


def test_interprocess_scale_down_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import _entry, free_port

    root = tempfile.mkdtemp()
    ctx = mp.get_context("spawn")
    qo, qn = ctx.Queue(), ctx.Queue()
    port = free_port()
    old = [ctx.Process(target=_entry, args=(r, 2, port, _old, (root,), qo, "nccl")) for r in range(2)]
    for p in old:
        p.start()
    newp = ctx.Process(target=_new, args=(root, qn))
    newp.start()
    status, val = qn.get(timeout=300)
    res = [qo.get(timeout=300) for _ in range(2)]
    newp.join(timeout=60)
    for p in old:
        p.join(timeout=60)
    assert status == "ok", val
    assert val is True
    assert all(r[1] == "ok" for r in res), res
