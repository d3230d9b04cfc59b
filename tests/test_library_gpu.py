"""``torch.ops.emb.*`` on a B200 runs the same kernels as the extension calls."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ops_match_extension():
    import elasticmegatron_b200.ops.library  # noqa: F401
    from elasticmegatron_b200.ops.native import ext

    torch.manual_seed(0)
    a = torch.randn(512, 256, device="cuda").bfloat16()
    b = torch.randn(384, 256, device="cuda").bfloat16()
    assert torch.equal(torch.ops.emb.gemm(a, b, False, True), ext().gemm(a, b, False, True))
    w = torch.randn(256, device="cuda").bfloat16()
    y, r = torch.ops.emb.rmsnorm_fwd(a, w, 1e-5)
    y2, r2 = ext().rmsnorm_fwd(a, w, 1e-5)
    assert torch.equal(y, y2) and torch.equal(r, r2)
    h = torch.randn(64, 512, device="cuda").bfloat16()
    assert torch.equal(torch.ops.emb.swiglu_fwd(h), ext().swiglu_fwd(h))
