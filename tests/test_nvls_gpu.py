"""All-reduce over NVSwitch multicast (multimem) and over peer memory on two GPUs: equal to NCCL's all-reduce bit
for bit (a sum of two fp32 values does not depend on its order), across chunk boundaries and odd lengths, and as
the Group-ZeRO gradient reduction inside training."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _allreduce(rank, world, kind):
    import torch
    import torch.distributed as dist

    from elasticmegatron_b200.parallel import nvls

    g = dist.new_group(list(range(world)))
    r = nvls.SymmetricAllReduce(g, torch.device("cuda", rank), chunk_bytes=1 << 20, force_p2p=kind == "p2p")
    out = {"kind": r.kind}
    ok = []
    for n in (1, 3, 4, 1000, 262144, 262147, 3 * 262144 + 5):  # last ones cross the 1 MiB chunk
        gen = torch.Generator(device="cuda").manual_seed(1000 * rank + n)
        x = torch.randn(n, device="cuda", generator=gen)
        ref = x.clone()
        dist.all_reduce(ref, group=g)
        r.all_reduce_(x)
        torch.cuda.synchronize()
        ok.append(bool(torch.equal(x, ref)))
    out["ok"] = ok
    from elasticmegatron_b200.ops.native import ext

    out["err"] = int(ext().comm_error_flag())
    return out


@pytest.mark.parametrize("kind", ["nvls", "p2p"])
def test_symmetric_all_reduce_matches_nccl(kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    res = run_distributed(_allreduce, 2, kind, backend="nccl")
    for rank in (0, 1):
        assert res[rank]["err"] == 0
        assert all(res[rank]["ok"]), res[rank]
    if kind == "p2p":
        assert res[0]["kind"] == "p2p"
    print("reducer:", res[0]["kind"])


def _group_zero_train(rank, world, nvls_mode):
    """Two optimizer instances on two GPUs (each GPU a full replica): the cross-instance gradient reduction runs
    through the symmetric all-reduce (or NCCL with EMB_NVLS=0)."""
    import os

    import torch
    os.environ["EMB_NVLS"] = nvls_mode
    torch.cuda.set_device(rank)
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState
    from elasticmegatron_b200.transfer.validate import state_checksum

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, ffn_hidden_size=512, vocab_size=1000,
                      seq_length=128, params_dtype="bf16", make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4, lr=3e-3)))
    S = ParallelStrategy(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                         num_distributed_optimizer_instances=2)
    create_all_groups([S])
    ts = TrainingState(S)
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    losses = [train_step(ts, it)["loss"] for _ in range(3)]
    from elasticmegatron_b200.parallel import nvls

    kinds = sorted(r.kind for r in nvls._CACHE.values())
    return losses, state_checksum(ts, None), kinds


def test_group_zero_training_nvls_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    nccl = run_distributed(_group_zero_train, 2, "0", backend="nccl")
    mine = run_distributed(_group_zero_train, 2, "nvls", backend="nccl")
    assert nccl[0][2] == [] and len(mine[0][2]) == 1  # the baseline used NCCL, the other run a reducer
    for r in (0, 1):
        assert mine[r][0] == nccl[r][0]
        assert mine[r][1] == nccl[r][1]
