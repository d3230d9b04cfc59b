"""Context parallelism on the native attention kernels (two GPUs): the all-gather, ring and Ulysses variants
against causal attention of the unsplit sequence in fp32 (outputs and gradients), and the LSE merge kernel
against its fp32 formula on one GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_attn_merge_matches_formula():
    from elasticmegatron_b200.ops.native import ext

    torch.manual_seed(0)
    s, b, H = 256, 2, 4
    out = torch.randn(s, b, H, 128, device="cuda")
    lse = torch.randn(b, H, s, device="cuda")
    lse[0, 0, :5] = float("-inf")  # rows with no block yet take the block's values
    o_b = torch.randn(s, b, H * 128, device="cuda").bfloat16()
    l_b = torch.randn(b, H, s, device="cuda")
    l_b[1, 2, 7:9] = float("-inf")  # fully masked block rows leave the row alone
    l_n = torch.logaddexp(lse, l_b)
    w0 = torch.exp(lse - l_n).permute(2, 0, 1)[..., None]
    w1 = torch.exp(l_b - l_n).permute(2, 0, 1)[..., None]
    ref = out * w0 + o_b.float().view(s, b, H, 128) * w1
    ext().attn_merge(out, lse, o_b, l_b)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(lse, l_n, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("causal", [True, False])
def test_flash_bwd_blocks(causal):
    """The backward kernel with a given (final) log-sum-exp, causal and not: the per-block call of CP."""
    from elasticmegatron_b200.ops import reference as ref
    from elasticmegatron_b200.ops.native import ext

    torch.manual_seed(1)
    s, b, G, hpg = 256, 1, 2, 2
    qkv = torch.randn(s, b, G, hpg + 2, 128, device="cuda").bfloat16()
    dO = torch.randn(s, b, G * hpg * 128, device="cuda").bfloat16()
    o, lse = ext().attn_fwd(qkv, hpg, causal)
    g = ext().attn_bwd(dO, qkv, o, lse, hpg, causal)
    torch.cuda.synchronize()
    x = qkv.float().requires_grad_(True)
    q = x[:, :, :, :hpg].reshape(s, b, G * hpg, 128).permute(1, 2, 0, 3)
    k, v = x[:, :, :, hpg].permute(1, 2, 0, 3), x[:, :, :, hpg + 1].permute(1, 2, 0, 3)
    y, _ = ref.attention_fwd(q, k, v, causal=causal)
    y = y.permute(2, 0, 1, 3).reshape(s, b, -1)
    (gr,) = torch.autograd.grad(y, x, dO.float())
    scale = gr.abs().max().item()
    torch.testing.assert_close(g.float(), gr, atol=3e-2 * max(1.0, scale / 4), rtol=5e-2)


def _cp_native(rank, world, hpg):
    import torch
    import torch.distributed as dist

    from elasticmegatron_b200.ops import reference as ref
    from elasticmegatron_b200.parallel.context_parallel import (cp_attention, cp_ring_attention,
                                                                cp_ulysses_attention)

    G, d, b, c = 2, 128, 2, 256
    S = 2 * world * c
    gen = torch.Generator(device="cuda").manual_seed(11)
    full = torch.randn(S, b, G, hpg + 2, d, generator=gen, device="cuda").bfloat16()
    dfull = torch.randn(S, b, G * hpg * d, generator=gen, device="cuda").bfloat16()
    idx = torch.cat([torch.arange(rank * c, (rank + 1) * c),
                     torch.arange((2 * world - 1 - rank) * c, (2 * world - rank) * c)]).cuda()
    # fp32 oracle: causal attention of the whole sequence
    F = full.float().requires_grad_()
    q = F[:, :, :, :hpg].reshape(S, b, G * hpg, d).permute(1, 2, 0, 3)
    k, v = F[:, :, :, hpg].permute(1, 2, 0, 3), F[:, :, :, hpg + 1].permute(1, 2, 0, 3)
    o, _ = ref.attention_fwd(q, k, v, causal=True)
    o = o.permute(2, 0, 1, 3).reshape(S, b, -1)
    (o * dfull.float()).sum().backward()
    o_ref, g_ref = o[idx].detach(), F.grad[idx]
    out = {}
    for name, fn in (("all_gather", cp_attention), ("p2p", cp_ring_attention), ("a2a", cp_ulysses_attention)):
        x = full[idx].clone().requires_grad_()
        y = fn(x, hpg, dist.group.WORLD, rank, world)
        y.backward(dfull[idx])
        torch.cuda.synchronize()
        out[name] = ((y.float() - o_ref).abs().max().item(), (x.grad.float() - g_ref).abs().max().item(),
                     g_ref.abs().max().item())
    from elasticmegatron_b200.ops.native import ext

    out["err"] = (int(ext().attn_error_flag()), int(ext().attn_bwd_error_flag()))
    return out


@pytest.mark.parametrize("hpg", [1, 2])
def test_cp2_native_matches_unsplit_attention(hpg):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from dist_utils import run_distributed

    res = run_distributed(_cp_native, 2, hpg, backend="nccl")
    for r in res:
        assert r["err"] == (0, 0)
        for name in ("all_gather", "p2p", "a2a"):
            fwd, bwd, scale = r[name]
            assert fwd < 2e-2, (name, r)
            assert bwd < 3e-2 * max(1.0, scale / 4), (name, r)
