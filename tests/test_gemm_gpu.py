"""tcgen05 GEMM against an fp32 torch reference, for the fprop / dgrad / wgrad operand layouts."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ext():
    from elasticmegatron_b200.ops.native import ext

    return ext()


SHAPES = [(128, 256, 64), (256, 512, 128), (296, 520, 200), (1024, 4096, 4096), (4096, 1024, 512), (8, 8, 8),
          (4096, 4096, 256), (2560, 2304, 128), (2600, 2200, 136),
          (136, 264, 72)]


@pytest.mark.parametrize("variant", [1, 2, 3])
@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("layout", ["fprop", "dgrad", "wgrad"])
def test_gemm_layouts(M, N, K, layout, variant):
    torch.manual_seed(0)
    dev = "cuda"
    if layout == "fprop":  # a [M,K], b [N,K], trans_b
        a = torch.randn(M, K, device=dev).bfloat16()
        b = torch.randn(N, K, device=dev).bfloat16()
        out = _ext().gemm_tc(a, b, False, True, variant=variant)
        exp = a.float() @ b.float().t()
    elif layout == "dgrad":  # a [M,K], b [K,N]
        a = torch.randn(M, K, device=dev).bfloat16()
        b = torch.randn(K, N, device=dev).bfloat16()
        out = _ext().gemm_tc(a, b, False, False, variant=variant)
        exp = a.float() @ b.float()
    else:  # a [K,M] (trans_a), b [K,N]; accumulate into fp32
        a = torch.randn(K, M, device=dev).bfloat16()
        b = torch.randn(K, N, device=dev).bfloat16()
        c = torch.ones(M, N, device=dev)
        out = _ext().gemm_tc(a, b, True, False, c, True, variant=variant)
        exp = a.float().t() @ b.float() + 1
    torch.cuda.synchronize()
    tol = 2e-2 * (K ** 0.5)
    torch.testing.assert_close(out.float(), exp, atol=tol, rtol=2e-2)


def test_gemm_fp32_out_store():
    a = torch.randn(256, 128, device="cuda").bfloat16()
    b = torch.randn(512, 128, device="cuda").bfloat16()
    c = torch.full((256, 512), 7.0, device="cuda")
    _ext().gemm_tc(a, b, False, True, c, False)
    torch.testing.assert_close(c, a.float() @ b.float().t(), atol=0.3, rtol=2e-2)


def test_gemm_unaligned_falls_back():
    """Operands whose leading dimension breaks the 16-byte TMA stride rule take the library path."""
    a = torch.randn(200, 300, device="cuda").bfloat16()
    b = torch.randn(200, 520, device="cuda").bfloat16()
    assert not _ext().gemm_tc_supported(a, b, True, False)
    out = _ext().gemm(a, b, True, False)
    torch.testing.assert_close(out.float(), a.float().t() @ b.float(), atol=0.5, rtol=2e-2)
