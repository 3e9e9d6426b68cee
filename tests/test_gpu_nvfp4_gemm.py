"""tcgen05 NVFP4 block-scaled GEMM against dequantise-then-multiply in fp32."""

import pytest
import torch

@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (256, 384, 512), (300, 200, 1024), (1024, 1024, 4096)])
def test_nvfp4_gemm_matches_dequantised_product(M, N, K):
    from llm_research_b200._ext import native
    from llm_research_b200.ops.quant import NVFP4Tensor, matmul_nvfp4

    torch.manual_seed(0)
    a = NVFP4Tensor.quantize(torch.randn(M, K, device="cuda", dtype=torch.bfloat16))
    b = NVFP4Tensor.quantize(torch.randn(N, K, device="cuda", dtype=torch.bfloat16))
    c = matmul_nvfp4(a, b)
    torch.cuda.synchronize()
    assert native().gemm_nvfp4_error(0) == 0
    ref = a.dequantize() @ b.dequantize().t()
    err = ((c.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err


def test_nvfp4_scale_swizzle_round_trip():
    from llm_research_b200.ops.quant import nvfp4_swizzle_scales

    M, KB = 200, 32
    s = torch.arange(M * KB, dtype=torch.int64).remainder(251).to(torch.uint8).view(M, KB)
    at = nvfp4_swizzle_scales(s).view(-1)
    for m in (0, 31, 32, 127, 128, 199):
        for j in (0, 3, 4, 31):
            blk, kb, jj = m // 128, j // 4, j % 4
            mm = m % 128
            off = (blk * (KB // 4) + kb) * 512 + 16 * (mm % 32) + 4 * (mm // 32) + jj
            assert int(at[off]) == int(s[m, j])
