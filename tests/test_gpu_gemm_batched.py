"""Batched tcgen05 GEMM with the axpby epilogue (row strides 16-byte aligned:
the last dimensions are multiples of 8), and the Newton-Schulz
iteration built on it, against fp32 PyTorch references."""

import pytest
import torch


@pytest.mark.gpu
@pytest.mark.parametrize("Bt,M,N,K", [(1, 128, 256, 64), (3, 200, 296, 136), (2, 512, 768, 1024)])
@pytest.mark.parametrize("b_mn", [False, True])
def test_gemm_batched_axpby(Bt, M, N, K, b_mn):
    from llm_research_b200._ext import native

    torch.manual_seed(0)
    A = torch.randn(Bt, M, K, device="cuda").bfloat16()
    B = torch.randn(Bt, K, N, device="cuda").bfloat16() if b_mn else torch.randn(Bt, N, K, device="cuda").bfloat16()
    D = torch.randn(Bt, M, N, device="cuda").bfloat16()
    C = torch.empty(Bt, M, N, device="cuda", dtype=torch.bfloat16)
    native().gemm_batched(A, B, b_mn, C, D, 0.5, -1.5)
    torch.cuda.synchronize()
    assert native().gemm_batched_error(0) == 0
    Bm = B.float() if b_mn else B.float().transpose(1, 2)
    ref = 0.5 * (A.float() @ Bm) - 1.5 * D.float()
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(4, 256, 256), (3, 512, 1408), (2, 2048, 5632)])
def test_newton_schulz_native_matches_fp32(shape):
    from llm_research_b200._ext import native
    from llm_research_b200.ops.optim import NS_A, NS_B, NS_C, newton_schulz

    torch.manual_seed(1)
    G = torch.randn(*shape, device="cuda")
    out = newton_schulz(G.bfloat16(), steps=5)
    torch.cuda.synchronize()
    assert native().gemm_batched_error(0) == 0
    X = G / (G.flatten(1).norm(dim=1).view(-1, 1, 1) + 1e-7)
    for _ in range(5):
        A = X @ X.transpose(1, 2)
        X = NS_A * X + (NS_B * A + NS_C * A @ A) @ X
    err = ((out.float() - X).norm() / X.norm()).item()
    assert err < 3e-2, err
