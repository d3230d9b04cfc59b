"""Native flash attention against the fp32 PyTorch reference on the fused QKV layout."""
import pytest
import torch

from elasticmegatron_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _ref(qkv, hpg, causal):
    s, b, G, _, d = qkv.shape
    x = qkv.float()
    q = x[:, :, :, :hpg].reshape(s, b, G * hpg, d).permute(1, 2, 0, 3)
    k = x[:, :, :, hpg].permute(1, 2, 0, 3)
    v = x[:, :, :, hpg + 1].permute(1, 2, 0, 3)
    o, lse = ref.attention_fwd(q, k, v, causal=causal)
    return o.permute(2, 0, 1, 3).reshape(s, b, -1), lse


@pytest.mark.parametrize("s,b,G,hpg", [(128, 1, 1, 1), (256, 2, 2, 2), (512, 1, 4, 1), (384, 2, 1, 4)])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_fwd(s, b, G, hpg, causal):
    from elasticmegatron_b200.ops.native import ext

    torch.manual_seed(0)
    qkv = torch.randn(s, b, G, hpg + 2, 128, device="cuda").bfloat16()
    o, lse = ext().attn_fwd(qkv, hpg, causal)
    torch.cuda.synchronize()
    assert ext().attn_error_flag() == 0
    o_ref, lse_ref = _ref(qkv, hpg, causal)
    torch.testing.assert_close(o.float(), o_ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, lse_ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("s,b,G,hpg", [(128, 1, 1, 1), (256, 2, 2, 2), (384, 1, 1, 4)])
def test_flash_bwd(s, b, G, hpg):
    from elasticmegatron_b200.ops.native import ext

    torch.manual_seed(0)
    qkv = torch.randn(s, b, G, hpg + 2, 128, device="cuda").bfloat16()
    dO = torch.randn(s, b, G * hpg * 128, device="cuda").bfloat16()
    o, lse = ext().attn_fwd(qkv, hpg, True)
    dqkv = ext().attn_bwd(dO, qkv, o, lse, hpg, True)
    torch.cuda.synchronize()
    assert ext().attn_bwd_error_flag() == 0
    x = qkv.float().requires_grad_(True)
    o_ref, _ = _ref(x, hpg, True)
    (g,) = torch.autograd.grad(o_ref, x, dO.float())
    scale = g.abs().max().item()
    torch.testing.assert_close(dqkv.float(), g, atol=3e-2 * max(1.0, scale / 4), rtol=5e-2)


def test_attention_autograd_native_path():
    """The model's attention op runs the native kernels on CUDA for head dim 128."""
    from elasticmegatron_b200.ops import functional as F_
    from elasticmegatron_b200.ops.native import launch_count

    import os

    os.environ["EMB_NATIVE_ATTENTION"] = "1"
    torch.manual_seed(0)
    qkv = torch.randn(256, 1, 2, 4, 128, device="cuda").bfloat16().requires_grad_(True)
    n0 = launch_count()
    y = F_.attention(qkv, 2)
    y.float().pow(2).sum().backward()
    torch.cuda.synchronize()
    os.environ.pop("EMB_NATIVE_ATTENTION")
    assert launch_count() - n0 >= 4
    x = qkv.detach().float().requires_grad_(True)
    o_ref, _ = _ref(x, 2, True)
    torch.testing.assert_close(y.float(), o_ref, atol=2e-2, rtol=2e-2)


def test_softmax_exp2_emulation_error_bound():
    """The FMA-pipe 2^x used for part of the softmax stays within 2e-4 relative of exp2 over the softmax's
    input range (scores minus the running max: at most +8, masked entries at -inf)."""
    from elasticmegatron_b200.ops.native import ext

    x = torch.cat([torch.linspace(-125.0, 8.0, 1 << 20, device="cuda"),
                   torch.rand(1 << 20, device="cuda") * -20.0, torch.tensor([0.5], device="cuda")])
    y = ext().attn_exp2_emulated(x)  # pairs through the packed form, the odd last element through the scalar one
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref).abs() / ref).max().item()
    assert rel < 2e-4, rel
    # inputs below -125 (and masked -inf) are clamped: a result below 2^-124, negligible next to the row max's 1
    z = ext().attn_exp2_emulated(torch.tensor([-float("inf"), -1000.0, -125.9], device="cuda"))
    assert (z >= 0).all() and (z < 2.0 ** -124).all()
