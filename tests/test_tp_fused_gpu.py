"""Fused TP collectives on two GPUs, against GEMM + NCCL references."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rs_case(rank, world):
    import torch.distributed as dist

    from elasticmegatron_b200.ops import tp_fused
    from elasticmegatron_b200.ops.native import ext

    g = dist.group.WORLD
    torch.manual_seed(1234)  # same operands on every rank, then rank-dependent scaling
    ok = True
    for trans_b, (M, N, K) in ((True, (1024, 768, 512)), (False, (512, 1024, 256)), (True, (4096, 4096, 1024))):
        a = (torch.randn(M, K, device="cuda") * (1 + rank)).bfloat16()
        b = torch.randn(*((N, K) if trans_b else (K, N)), device="cuda").bfloat16()
        full = ext().gemm_tc(a, b, False, trans_b)
        ref = torch.empty(M // world, N, device="cuda", dtype=torch.bfloat16)
        dist.reduce_scatter_tensor(ref, full, group=g)
        got = tp_fused.gemm_reduce_scatter(a, b, False, trans_b, g)
        torch.cuda.synchronize()
        ok &= torch.allclose(got.float(), ref.float(), atol=0.05 * (K ** 0.5), rtol=2e-2)
    # the buffers can be released (as before re-creating communicators) and are rebuilt on the next call
    tp_fused.release_buffers()
    got = tp_fused.gemm_reduce_scatter(a, b, False, trans_b, g)
    torch.cuda.synchronize()
    ok &= torch.allclose(got.float(), ref.float(), atol=0.05 * (K ** 0.5), rtol=2e-2)
    ok &= ext().comm_error_flag() == 0
    return bool(ok)


def _ag_case(rank, world):
    import torch.distributed as dist

    from elasticmegatron_b200.ops import tp_fused
    from elasticmegatron_b200.ops.native import ext

    g = dist.group.WORLD
    ok = True
    for trans_b, (R, N, K) in ((True, (512, 768, 512)), (False, (256, 1024, 256)), (True, (2048, 6144, 4096))):
        torch.manual_seed(rank)
        shard = torch.randn(R, K, device="cuda").bfloat16()
        torch.manual_seed(99)
        b = torch.randn(*((N, K) if trans_b else (K, N)), device="cuda").bfloat16()
        full = torch.empty(world * R, K, device="cuda", dtype=torch.bfloat16)
        dist.all_gather_into_tensor(full, shard, group=g)
        ref = ext().gemm_tc(full, b, False, trans_b)
        for _ in range(2):  # twice: the symmetric buffer and ready counters are reused
            got, gathered = tp_fused.all_gather_gemm(shard, b, trans_b, g)
            torch.cuda.synchronize()
            ok &= torch.equal(gathered, full)
            ok &= torch.allclose(got.float(), ref.float(), atol=1e-2, rtol=1e-2)
    ok &= ext().gemm_error_flag() == 0 and ext().comm_error_flag() == 0
    return bool(ok)


def test_fused_all_gather_gemm():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    assert all(run_distributed(_ag_case, 2, backend="nccl"))


def _tp_train(rank, world, fused):
    os.environ["EMB_FUSED_TP"] = "1" if fused else "0"
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=512, num_attention_heads=4, ffn_hidden_size=1024, vocab_size=1000,
                      seq_length=512, params_dtype="bf16", max_tensor_parallel_size=2, make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4)))
    s = ParallelStrategy(world_size=2, tensor_model_parallel_size=2, pipeline_model_parallel_size=1)
    create_all_groups([s])
    ts = TrainingState(s)
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    return [train_step(ts, it)["loss"] for _ in range(3)]


def test_fused_gemm_reduce_scatter():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    assert all(run_distributed(_rs_case, 2, backend="nccl"))


def test_tp2_training_fused_matches_nccl_path():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    a = run_distributed(_tp_train, 2, True, backend="nccl")[0]
    b = run_distributed(_tp_train, 2, False, backend="nccl")[0]
    torch.testing.assert_close(torch.tensor(a), torch.tensor(b), atol=2e-2, rtol=2e-3)


def test_sym_barrier_bounded_wait():
    """One GPU: a barrier whose 'peer' slot nobody writes gives up after its limit and reports the peer."""
    from elasticmegatron_b200.ops.native import ext

    own = torch.zeros(1024, dtype=torch.int32, device="cuda")
    fake_peer = torch.zeros(1024, dtype=torch.int32, device="cuda")
    sig = torch.tensor([own.data_ptr(), fake_peer.data_ptr()], dtype=torch.int64)
    ext().comm_clear_error()
    own[1] = 3  # the peer already reached epoch 3: epochs 1..3 pass at once
    for e in (1, 2, 3):
        ext().sym_barrier(sig, 0, e, 1000)
    torch.cuda.synchronize()
    assert ext().comm_error_flag() == 0
    assert int(fake_peer[0]) == 3  # our arrivals were stored into the peer's slot 0
    ext().sym_barrier(sig, 0, 4, 100)  # nobody stores epoch 4 into our slot 1
    torch.cuda.synchronize()
    assert ext().comm_error_flag() == 0x5001
    ext().comm_clear_error()
    assert ext().comm_error_flag() == 0
