"""Operator registrations (``torch.ops.emb.*``): shapes and dtypes from the fake implementations on meta tensors,
no GPU needed; CPU tensors have no kernel."""
import pytest
import torch


def test_fake_shapes_on_meta():
    import elasticmegatron_b200.ops.library  # noqa: F401  registers the operators

    ops = torch.ops.emb
    m = dict(device="meta", dtype=torch.bfloat16)
    a, b = torch.empty(64, 32, **m), torch.empty(48, 32, **m)
    assert ops.gemm(a, b, False, True).shape == (64, 48)
    assert ops.gemm(a.t(), b.t(), True, False).shape == (64, 48)
    w = torch.empty(3, 80, 32, **m)
    assert ops.gemm_grouped(torch.empty(256, 32, **m), w, True, torch.empty(2, device="meta", dtype=torch.int32)
                            ).shape == (256, 80)
    x, g = torch.empty(10, 256, **m), torch.empty(256, **m)
    y, rstd = ops.rmsnorm_fwd(x, g, 1e-5)
    assert y.shape == x.shape and rstd.shape == (10,) and rstd.dtype == torch.float32
    dx, dw = ops.rmsnorm_bwd(x, x, g, rstd)
    assert dx.shape == x.shape and dw.shape == (256,) and dw.dtype == torch.float32
    h = torch.empty(4, 7, 128, **m)
    assert ops.swiglu_fwd(h).shape == (4, 7, 64) and ops.swiglu_bwd(torch.empty(4, 7, 64, **m), h).shape == h.shape
    qkv = torch.empty(16, 2, 4, 4, 64, **m)  # [s, b, groups, q-per-group + 2, d]
    c = torch.empty(16, 32, device="meta")
    assert ops.rope_fwd(qkv, c, c, 3, False).shape == qkv.shape
    o, lse = ops.attn_fwd(qkv, 2, True)
    assert o.shape == (16, 2, 4 * 2 * 64) and lse.shape == (2, 8, 16) and lse.dtype == torch.float32
    logits = torch.empty(9, 1000, **m)
    assert ops.ce_local_max(logits).shape == (9,)
    lab = torch.empty(9, device="meta", dtype=torch.long)
    assert ops.ce_local_stats(logits, lab, torch.empty(9, device="meta"), 0).shape == (2, 9)
    emb = torch.empty(1000, 256, **m)
    assert ops.embedding_fwd(torch.empty(3, 5, device="meta", dtype=torch.long), emb, 0).shape == (15, 256)


def test_cpu_tensors_have_no_kernel():
    import elasticmegatron_b200.ops.library  # noqa: F401

    with pytest.raises(NotImplementedError):
        torch.ops.emb.swiglu_fwd(torch.zeros(2, 16, dtype=torch.bfloat16))
