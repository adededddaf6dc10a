"""The weight-streaming GEMM (anemll_gemm) against an fp32 product of the same fp16/bf16 operands."""
import pytest
import torch

from tests.tolerance import assert_close

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("M,N,K", [(1, 2048, 4096), (128, 2048, 6144), (128, 12352, 2048), (64, 9216, 2048),
                                   (7, 200, 72), (128, 1000, 512), (200, 384, 1024), (33, 151936, 256)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemm_matches_fp32_product(M, N, K, dt):
    from anemll_b200 import dense
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).to(dt)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(dt)
    y = dense.gemm(x.to(DEV), w.to(DEV))
    ref = x.float() @ w.float().T
    # one rounding of the fp32 sum to the 8/11-bit mantissa of the output
    tol = 4e-3 if dt == torch.bfloat16 else 1e-3
    assert_close(y.float().cpu(), ref, f"gemm {M}x{N}x{K}", rel_l2=tol, max_abs=8 * tol * ref.abs().max().item())
    assert dense.gemm_device_error() == 0


def test_linear_routes_and_strided_rows():
    from anemll_b200 import dense
    g = torch.Generator().manual_seed(3)
    w = torch.randn(256, 512, generator=g).bfloat16().to(DEV)
    wide = torch.randn(4, 3, 1024, generator=g).bfloat16().to(DEV)
    x = wide[..., 256:768]  # rows 1024 elements apart
    y = dense.linear(x, w) if dense.SKINNY_ROWS >= 12 else dense.gemm(x.reshape(12, 512), w).view(4, 3, 256)
    assert y.shape == (4, 3, 256)
    ref = torch.nn.functional.linear(x.float(), w.float())
    assert_close(y.float(), ref, "linear", rel_l2=4e-3, max_abs=0.05 * ref.abs().max().item())
    big = torch.randn(300, 512, device=DEV).bfloat16()  # more rows than SKINNY_ROWS: torch's GEMM
    assert torch.equal(dense.linear(big, w), torch.nn.functional.linear(big, w))


def test_gemm_errors():
    from anemll_b200 import dense
    with pytest.raises(TypeError):
        dense.gemm(torch.zeros(2, 8, device=DEV), torch.zeros(8, 8, device=DEV))
    with pytest.raises(RuntimeError, match="CUDA"):
        dense.gemm(torch.zeros(2, 8).half(), torch.zeros(8, 8).half())
