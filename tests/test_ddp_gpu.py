"""Data parallelism on two GPUs: the bucketed gradient reduce-scatter left in flight during backward and the
parameter all-gathers left in flight until the next forward (overlap_grad_reduce / overlap_param_gather) give
bit-identical losses and parameters to the blocking order, and the peer-memory collectives (K6 / K7) give
bit-identical results to NCCL's (a sum of two fp32 values does not depend on its order)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _train(rank, world, overlap, peer=True):
    import os

    import torch
    torch.cuda.set_device(rank)
    os.environ["EMB_DP_PEER"] = "1" if peer else "0"
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState
    from elasticmegatron_b200.transfer.validate import state_checksum

    cfg = ModelConfig(num_layers=4, hidden_size=256, num_attention_heads=4, ffn_hidden_size=512, vocab_size=1000,
                      seq_length=128, params_dtype="bf16", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, overlap_grad_reduce=True,
                                               overlap_param_gather=overlap, ddp_bucket_size=200000)))
    S = ParallelStrategy(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1)
    create_all_groups([S])
    ts = TrainingState(S)
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    losses = [train_step(ts, it)["loss"] for _ in range(3)]
    # reading the whole arena waits for the in-flight gathers of the last step
    return losses, state_checksum(ts, None), len(ts.ddp._bucket_keys), ts.ddp.peer is not None


def test_overlapped_param_gather_matches_blocking():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    a = run_distributed(_train, 2, False, backend="nccl")
    b = run_distributed(_train, 2, True, backend="nccl")
    assert a[0][2] > 1  # several buckets, so the per-bucket waits matter
    assert a[0][0] == b[0][0] and a[1][0] == b[1][0]
    assert a[0][1] == b[0][1] and a[1][1] == b[1][1]


def test_peer_memory_dp_collectives_match_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    nccl = run_distributed(_train, 2, True, False, backend="nccl")
    peer = run_distributed(_train, 2, True, True, backend="nccl")
    assert peer[0][3] and not nccl[0][3]  # the peer path ran, and the baseline did not
    assert peer[0][0] == nccl[0][0] and peer[1][0] == nccl[1][0]
    assert peer[0][1] == nccl[0][1] and peer[1][1] == nccl[1][1]
