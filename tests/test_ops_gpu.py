"""Numerics of the native sm_100a kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

from elasticmegatron_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _ext():
    from elasticmegatron_b200.ops.native import ext

    return ext()


def _close(a, b, atol, rtol):
    torch.testing.assert_close(a.float(), b.float(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("T,H", [(257, 512), (1024, 4096), (64, 5120)])
def test_rmsnorm(T, H):
    torch.manual_seed(0)
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    y, rstd = _ext().rmsnorm_fwd(x, w, 1e-5)
    y_ref, rstd_ref = ref.rmsnorm_fwd(x.float(), w.float(), 1e-5)
    _close(y, y_ref, 2e-2, 2e-2)
    _close(rstd, rstd_ref, 1e-4, 1e-4)
    dy = torch.randn(T, H, device="cuda").bfloat16()
    dx, dw = _ext().rmsnorm_bwd(dy, x, w, rstd)
    dx_ref, dw_ref = ref.rmsnorm_bwd(dy.float(), x.float(), w.float(), rstd_ref)
    _close(dx, dx_ref, 3e-2, 3e-2)
    _close(dw, dw_ref, 5e-2 * math.sqrt(T / 64), 1e-2)
    acc = torch.ones(H, device="cuda")
    _ext().rmsnorm_bwd(dy, x, w, rstd, acc)
    _close(acc, dw_ref + 1, 5e-2 * math.sqrt(T / 64), 1e-2)


@pytest.mark.parametrize("T,H", [(7, 512), (300, 4096)])
def test_add_rmsnorm_fused(T, H):
    """Residual add fused into RMSNorm (forward) and the residual gradient added in the norm's backward, against
    the fp32 reference of the unfused pair."""
    torch.manual_seed(1)
    x = torch.randn(T, H, device="cuda").bfloat16()
    o = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    h, y, rstd = _ext().add_rmsnorm_fwd(x, o, w, 1e-5)
    h_ref = (x.float() + o.float()).bfloat16().float()  # the residual stream is bf16
    y_ref, rstd_ref = ref.rmsnorm_fwd(h_ref, w.float(), 1e-5)
    _close(h, h_ref, 1e-6, 1e-6)
    _close(y, y_ref, 2e-2, 2e-2)
    _close(rstd, rstd_ref, 1e-4, 1e-4)
    dy = torch.randn(T, H, device="cuda").bfloat16()
    dh = torch.randn(T, H, device="cuda").bfloat16()
    dx, dw = _ext().rmsnorm_bwd(dy, h, w, rstd, None, dh)
    dx_ref, dw_ref = ref.rmsnorm_bwd(dy.float(), h_ref, w.float(), rstd_ref)
    _close(dx, dx_ref + dh.float(), 3e-2, 3e-2)
    _close(dw, dw_ref, 5e-2 * math.sqrt(T / 64), 1e-2)


def test_add_rmsnorm_autograd_matches_unfused():
    from elasticmegatron_b200.ops import functional as F_

    torch.manual_seed(2)
    T, H = 256, 1024
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_(True)
    o = torch.randn(T, H, device="cuda").bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_(True)
    h, y = F_.add_rmsnorm(x, o, w, 1e-5)
    (h.float().sum() + (y.float() ** 2).sum()).backward()
    xr, orr, wr = (t.detach().float().requires_grad_(True) for t in (x, o, w))
    hr = xr + orr
    yr = hr * torch.rsqrt(hr.pow(2).mean(-1, keepdim=True) + 1e-5) * wr
    (hr.sum() + (yr ** 2).sum()).backward()
    _close(x.grad, xr.grad, 5e-2, 3e-2)
    _close(o.grad, orr.grad, 5e-2, 3e-2)
    _close(w.grad, wr.grad, 2.0, 3e-2)


def test_swiglu():
    torch.manual_seed(0)
    h = torch.randn(333, 2 * 1376, device="cuda").bfloat16()
    _close(_ext().swiglu_fwd(h), ref.swiglu_fwd(h.float()), 2e-2, 2e-2)
    dy = torch.randn(333, 1376, device="cuda").bfloat16()
    _close(_ext().swiglu_bwd(dy, h), ref.swiglu_bwd(dy.float(), h.float()), 3e-2, 3e-2)


@pytest.mark.parametrize("inverse", [False, True])
def test_rope(inverse):
    torch.manual_seed(0)
    s, b, G, hpg, d = 64, 2, 4, 2, 128
    qkv = torch.randn(s, b, G, hpg + 2, d, device="cuda").bfloat16()
    cos, sin = ref.rope_cos_sin(torch.arange(s), d, 10000.0)
    cos, sin = cos.cuda(), sin.cuda()
    out = _ext().rope_fwd(qkv, cos, sin, hpg + 1, inverse)
    exp = qkv.float().clone()
    x = exp[:, :, :, :hpg + 1].reshape(s, b, -1, d)
    exp[:, :, :, :hpg + 1] = ref.rope_apply(x, cos, sin, inverse).view(s, b, G, hpg + 1, d)
    _close(out, exp, 2e-2, 2e-2)


def test_cross_entropy_pieces():
    torch.manual_seed(0)
    T, V, vs = 300, 1024, 512
    logits = (3 * torch.randn(T, V, device="cuda")).bfloat16()
    labels = torch.randint(0, 2048, (T,), device="cuda")
    lmax = _ext().ce_local_max(logits)
    _close(lmax, logits.float().max(-1).values, 0, 0)
    st = _ext().ce_local_stats(logits, labels, lmax, vs)
    lf = logits.float()
    se = torch.exp(lf - lmax[:, None]).sum(-1)
    _close(st[0], se, 1e-3, 1e-4)
    loc = labels - vs
    inr = (loc >= 0) & (loc < V)
    tgt = torch.where(inr, lf.gather(1, loc.clamp(0, V - 1)[:, None]).squeeze(1) - lmax, torch.zeros_like(lmax))
    _close(st[1], tgt, 1e-5, 1e-5)
    dl = torch.rand(T, device="cuda")
    d = _ext().ce_bwd(logits, labels, lmax, se, dl, vs)
    p = torch.exp(lf - lmax[:, None]) / se[:, None]
    rows = torch.nonzero(inr).squeeze(1)
    p[rows, loc[rows]] -= 1
    _close(d, p * dl[:, None], 1e-2, 1e-2)


def test_embedding():
    torch.manual_seed(0)
    V, H, T, vs = 100, 256, 500, 50
    w = torch.randn(V, H, device="cuda").bfloat16()
    ids = torch.randint(0, 200, (T,), device="cuda")
    out = _ext().embedding_fwd(ids, w, vs)
    loc = ids - vs
    m = (loc >= 0) & (loc < V)
    exp = torch.zeros(T, H, device="cuda")
    exp[m] = w.float()[loc[m]]
    _close(out, exp, 0, 0)
    dy = torch.randn(T, H, device="cuda").bfloat16()
    tgt = torch.zeros(V, H, device="cuda")
    _ext().embedding_bwd(ids, dy, tgt, vs)
    ref_t = torch.zeros(V, H, device="cuda").index_add_(0, loc[m], dy.float()[m])
    _close(tgt, ref_t, 1e-4, 1e-4)


def test_adam_and_sumsq():
    torch.manual_seed(0)
    n = 70000
    O = torch.randn(3, n, device="cuda")
    O[2].abs_()
    G = torch.randn(n, device="cuda")
    P = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    chunks = torch.tensor([[0, 0, 40000, 1, 1], [40000, 40000, 30000, 0, 0]], device="cuda")
    sq = _ext().seg_sumsq(G, chunks)
    _close(sq, (G[:40000].double() ** 2).sum().float().reshape(1), 1e-2, 1e-5)
    O_ref = O.clone()
    _ext().adam_segments(O, G, P, chunks, 1e-3, 0.9, 0.95, 1e-8, 0.1, 3, 0.5, 1.0, sq)
    norm = math.sqrt(float(sq)) * 0.5
    clip = min(1.0, 1.0 / (norm + 1e-6))
    for a, o, k, wd in ((0, 0, 40000, 0.1), (40000, 40000, 30000, 0.0)):
        m, e1, e2 = O_ref[0, o:o + k], O_ref[1, o:o + k], O_ref[2, o:o + k]
        ref.adam_step(m, e1, e2, G[a:a + k], 1e-3, 0.9, 0.95, 1e-8, wd, 3, 0.5 * clip)
    _close(O, O_ref, 1e-6, 1e-5)
    _close(P, O_ref[0], 1e-2, 1e-2)


@pytest.mark.parametrize("T,H", [(9, 512), (300, 4096)])
def test_layernorm_native(T, H):
    """Native LayerNorm forward / backward against the fp32 PyTorch reference."""
    from elasticmegatron_b200.ops import functional as F_

    torch.manual_seed(3)
    x = torch.randn(T, H, device="cuda").bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_(True)
    b = (0.1 * torch.randn(H, device="cuda")).bfloat16().requires_grad_(True)
    n0 = _ext().launch_count()
    y = F_.layernorm(x, w, b, 1e-5)
    dy = torch.randn(T, H, device="cuda").bfloat16()
    y.backward(dy)
    assert _ext().launch_count() - n0 >= 3  # the native kernels ran
    xr, wr, br = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    yr = torch.nn.functional.layer_norm(xr, (H,), wr, br, 1e-5)
    yr.backward(dy.float())
    _close(y, yr, 2e-2, 2e-2)
    _close(x.grad, xr.grad, 3e-2, 3e-2)
    _close(w.grad, wr.grad, 5e-2 * math.sqrt(T / 8), 2e-2)
    _close(b.grad, br.grad, 5e-2 * math.sqrt(T / 8), 2e-2)


def test_layernorm_model_trains_on_gpu():
    """The reference demo's LayerNorm model (weight + bias per norm) takes training steps on one GPU through the
    native kernels: finite losses near ln(vocab) on the uniform synthetic tokens, and the weights move."""
    from elasticmegatron_b200.config import Args, ModelConfig, TrainConfig, set_args
    from elasticmegatron_b200.parallel.strategy import ParallelStrategy
    from elasticmegatron_b200.runtime.data import DataloaderState
    from elasticmegatron_b200.runtime.train import train_step
    from elasticmegatron_b200.runtime.training_state import TrainingState

    cfg = ModelConfig(num_layers=2, hidden_size=256, num_attention_heads=4, ffn_hidden_size=512, vocab_size=1000,
                      seq_length=128, params_dtype="bf16", normalization="LayerNorm",
                      make_vocab_size_divisible_by=8)
    set_args(Args(model=cfg, train=TrainConfig(micro_batch_size=2, global_batch_size=4, lr=3e-3)))
    ts = TrainingState(ParallelStrategy(world_size=1, tensor_model_parallel_size=1, pipeline_model_parallel_size=1))
    ts.init_weights(0)
    it = DataloaderState.build_iterators(ts, 0)[0]
    n0 = _ext().launch_count()
    p0 = ts.param_flat.clone()
    losses = [train_step(ts, it)["loss"] for _ in range(3)]
    assert _ext().launch_count() > n0
    assert all(5.0 < l < 9.0 for l in losses), losses
    assert not torch.equal(p0, ts.param_flat)
