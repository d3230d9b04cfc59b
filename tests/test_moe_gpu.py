"""MoE kernels on one B200 against plain PyTorch fp32 references: router, token layout, grouped GEMM, and the whole
native MoE layer against the per-expert PyTorch path inside a training step."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    from elasticmegatron_b200.ops.native import ext

    return ext()


@pytest.mark.parametrize("T,E,k", [(1000, 8, 2), (513, 64, 4), (64, 3, 1)])
def test_router_forward_backward(T, E, k):
    torch.manual_seed(0)
    logits = torch.randn(T, E, device="cuda") * 2
    top, probs, counts, part = _ext().moe_router_fwd(logits, k)
    ref_v, ref_i = logits.topk(k, dim=-1)
    assert torch.equal(top.long(), ref_i)
    torch.testing.assert_close(probs, torch.softmax(ref_v, -1), atol=1e-6, rtol=1e-5)
    assert torch.equal(counts.long(), torch.bincount(ref_i.reshape(-1), minlength=E))
    torch.testing.assert_close(part.sum(0), torch.softmax(logits, -1).sum(0), atol=1e-3, rtol=1e-5)
    # backward: probs and score sums against autograd of the fp32 reference
    lg = logits.clone().requires_grad_(True)
    pv = torch.softmax(lg.gather(1, ref_i), -1)
    ss = torch.softmax(lg, -1).sum(0)
    dp, ds = torch.randn_like(pv), torch.randn(E, device="cuda")
    (pv * dp).sum().backward(retain_graph=True)
    (ss * ds).sum().backward()
    got = _ext().moe_router_bwd(logits, top, probs, dp.contiguous(), ds.contiguous())
    torch.testing.assert_close(got, lg.grad, atol=1e-5, rtol=1e-4)


def test_layout_scatter_gather():
    torch.manual_seed(1)
    T, k, E, H = 700, 2, 8, 256
    gid = torch.randint(0, E, (T * k,), device="cuda", dtype=torch.int32)
    gid[:50] = 3  # an uneven segment
    counts = torch.bincount(gid.long(), minlength=E).int()
    cap = (T * k + E * 127 + 127) // 128 * 128
    pos, seg, tiles = _ext().moe_layout(gid, counts, cap, 128)
    seg_ref = [0]
    for c in counts.tolist():
        seg_ref.append(seg_ref[-1] + (c + 127) // 128 * 128)
    assert seg.tolist() == seg_ref
    order = torch.argsort(gid.long(), stable=True)
    exp_pos = torch.empty_like(order)
    for e in range(E):
        idx = order[gid[order] == e]
        exp_pos[idx] = seg_ref[e] + torch.arange(idx.numel(), device="cuda")
    assert torch.equal(pos.long(), exp_pos)
    tl = tiles.tolist()
    for i, g in enumerate(tl):
        row = 128 * i
        want = next((e for e in range(E) if seg_ref[e] <= row < seg_ref[e + 1]), -1)
        assert g == want
    x = torch.randn(T, H, device="cuda").bfloat16()
    xp = _ext().moe_scatter(x, k, pos, None, seg, counts, cap)
    assert torch.equal(xp[pos.long()], x.repeat_interleave(k, 0))
    for e in range(E):  # padding rows of each segment are zero
        assert (xp[seg_ref[e] + int(counts[e]):seg_ref[e + 1]] == 0).all()
    w = torch.rand(T * k, device="cuda")
    y = _ext().moe_gather(xp, pos, w, T, k)
    ref = (x.float().repeat_interleave(k, 0) * w[:, None]).view(T, k, H).sum(1)
    torch.testing.assert_close(y.float(), ref, atol=2e-2, rtol=1e-2)
    d = _ext().moe_row_dot(x, k, xp, pos)
    torch.testing.assert_close(d, (x.float().repeat_interleave(k, 0) ** 2).sum(1), atol=1e-1, rtol=1e-3)


@pytest.mark.parametrize("G,K,N", [(4, 512, 768), (3, 256, 1024)])
def test_grouped_gemm_fprop_dgrad_wgrad(G, K, N):
    torch.manual_seed(2)
    counts = torch.tensor([300, 0, 129, 64][:G] + [5] * max(0, G - 4), device="cuda", dtype=torch.int32)
    R = int(counts.sum())
    gid = torch.repeat_interleave(torch.arange(G, device="cuda", dtype=torch.int32), counts.long())
    cap = (R + G * 127 + 127) // 128 * 128
    pos, seg, tiles = _ext().moe_layout(gid, counts, cap, 128)
    x = (torch.randn(R, K, device="cuda") * 0.5).bfloat16()
    xp = _ext().moe_scatter(x, 1, pos, None, seg, counts, cap)
    w = (torch.randn(G, N, K, device="cuda") * 0.05).bfloat16()
    y = _ext().gemm_grouped(xp, w, True, tiles)
    o = 0
    for g in range(G):
        n = int(counts[g])
        ref = x[o:o + n].float() @ w[g].float().t()
        torch.testing.assert_close(y[pos[o:o + n].long()].float(), ref, atol=3e-2, rtol=2e-2)
        o += n
    # dgrad: dx = dy @ W[g]
    dy = (torch.randn(R, N, device="cuda") * 0.5).bfloat16()
    dyp = _ext().moe_scatter(dy, 1, pos, None, seg, counts, cap)
    dx = _ext().gemm_grouped(dyp, w, False, tiles)
    o = 0
    for g in range(G):
        n = int(counts[g])
        ref = dy[o:o + n].float() @ w[g].float()
        torch.testing.assert_close(dx[pos[o:o + n].long()].float(), ref, atol=3e-2, rtol=2e-2)
        o += n
    # wgrad: out[g] += dy_g^T x_g (fp32 accumulate into an existing buffer)
    base = torch.randn(G, N, K, device="cuda")
    out = base.clone()
    _ext().gemm_grouped_wgrad(dyp, xp, seg, out, True)
    o = 0
    for g in range(G):
        n = int(counts[g])
        ref = base[g] + dy[o:o + n].float().t() @ x[o:o + n].float()
        torch.testing.assert_close(out[g], ref, atol=5e-2, rtol=1e-2)
        o += n
    assert _ext().gemm_error_flag() == 0


def _moe_train(native: bool, ep: int = 1):
    os.environ["EMB_NATIVE_MOE"] = "1" if native else "0"
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, num_query_groups=2, ffn_hidden_size=512,
                      vocab_size=1000, seq_length=256, params_dtype="bf16", make_vocab_size_divisible_by=8,
                      num_experts=8, moe_ffn_hidden_size=256, moe_router_topk=2)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4, lr=1e-3)))
    ts = TrainingState(ParallelStrategy(world_size=1, tensor_model_parallel_size=1, pipeline_model_parallel_size=1))
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    out = []
    for _ in range(3):
        r = train_step(ts, it)
        out.append((r["loss"], float(r["grad_norm"])))
    return out


def test_native_moe_training_matches_torch_path():
    a = _moe_train(True)
    b = _moe_train(False)
    os.environ.pop("EMB_NATIVE_MOE", None)
    for (la, ga), (lb, gb) in zip(a, b):
        assert abs(la - lb) <= 2e-3 * abs(lb), (a, b)
        assert abs(ga - gb) <= 2e-2 * abs(gb), (a, b)


def _moe_ep_train(rank, world, native, peer=True):
    os.environ["EMB_NATIVE_MOE"] = "1" if native else "0"
    os.environ["EMB_EP_PEER"] = "1" if peer else "0"
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.process_groups import create_all_groups
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, num_query_groups=2, ffn_hidden_size=512,
                      vocab_size=1000, seq_length=256, params_dtype="bf16", make_vocab_size_divisible_by=8,
                      num_experts=8, moe_ffn_hidden_size=256, moe_router_topk=2, max_tensor_parallel_size=2)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=8, lr=1e-3)))
    s = ParallelStrategy(world_size=2, tensor_model_parallel_size=1, pipeline_model_parallel_size=1,
                         expert_model_parallel_size=2)
    create_all_groups([s])
    ts = TrainingState(s)
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    out = [train_step(ts, it)["loss"] for _ in range(3)]
    from elasticmegatron_b200.ops.native import ext

    assert ext().comm_error_flag() == 0
    return out


def test_native_moe_expert_parallel_matches_torch_path():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    a = run_distributed(_moe_ep_train, 2, True, backend="nccl")[0]
    b = run_distributed(_moe_ep_train, 2, False, backend="nccl")[0]
    torch.testing.assert_close(torch.tensor(a), torch.tensor(b), atol=1e-2, rtol=2e-3)


def test_ep_peer_dispatch_matches_nccl_all_to_all():
    """The peer-memory dispatch / combine gives the same training losses as NCCL all-to-all (same kernels around)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    a = run_distributed(_moe_ep_train, 2, True, True, backend="nccl")[0]
    b = run_distributed(_moe_ep_train, 2, True, False, backend="nccl")[0]
    torch.testing.assert_close(torch.tensor(a), torch.tensor(b), atol=1e-3, rtol=1e-4)


def _ep_plan_outlives_grow(rank, world):
    """Plan A pushes, plan B (more rows, all routed to rank 0's experts) grows the landing buffer, then plan A
    moves rows again, as the backward of an earlier layer does after a later layer's forward."""
    import torch.distributed as dist

    from elasticmegatron_b200.ops import ep_comm, tp_fused

    g = dist.new_group([0, 1])
    T, k, E, H = 256, 2, 4, 2048
    gen = torch.Generator(device="cuda").manual_seed(rank)

    def plan(top):
        counts = torch.bincount(top.reshape(-1), minlength=E).to(torch.int32)
        return ep_comm.EPPlan(g, top, counts, E // world, H)

    top_a = torch.randint(0, E, (T, k), device="cuda", generator=gen)
    top_b = torch.randint(0, E // world, (T, k), device="cuda", generator=gen)  # all to rank 0
    x = torch.randn(T, H, device="cuda", generator=gen).to(torch.bfloat16)
    a = plan(top_a)
    first = a.send_home(a.push(x, None, with_origin=True))
    half_a = a.land.half
    b = plan(top_b)
    b.send_home(b.push(x, None, with_origin=True))
    grown = a.land.half > half_a
    again = a.send_home(a.push(x, None, with_origin=True))
    want = x.repeat_interleave(k, 0)
    ok = bool(torch.equal(first, want)) and bool(torch.equal(again, want))
    tp_fused.release_buffers()
    return ok, grown


def test_ep_plan_survives_buffer_grow():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    res = run_distributed(_ep_plan_outlives_grow, 2, backend="nccl")
    assert all(ok for ok, _ in res) and any(grown for _, grown in res), res
