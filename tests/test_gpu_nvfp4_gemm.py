"""tcgen05 NVFP4 block-scaled GEMM against dequantise-then-multiply in fp32."""

import pytest
import torch

@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (256, 384, 512), (300, 200, 1024), (1024, 1024, 4096),
                                   (256, 512, 512), (300, 768, 1024)])
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


@pytest.mark.gpu
def test_nvfp4_linear_forward_backward_close_to_bf16():
    """The NVFP4 training linear (RNE forward, stochastic-rounding backward) against bf16."""
    from llm_research_b200.ops.linear import linear_precision, project

    torch.manual_seed(0)
    x = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(768, 1024, device="cuda") * 0.03).to(torch.bfloat16).requires_grad_()
    dy = torch.randn(512, 768, device="cuda", dtype=torch.bfloat16)
    y_ref = torch.nn.functional.linear(x.float(), w.float())
    gx_ref, gw_ref = torch.autograd.grad(y_ref, (x, w), dy.float())
    with linear_precision("nvfp4"):
        y = project(x, w)
    gx, gw = torch.autograd.grad(y, (x, w), dy)
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()
    assert rel(y, y_ref) < 0.15
    assert rel(gx, gx_ref) < 0.2
    assert rel(gw, gw_ref) < 0.2


@pytest.mark.gpu
def test_hlrt_trains_with_nvfp4_linears():
    from genesis.model import HLRT, HLRTConfig
    from llm_research_b200.ops.linear import linear_precision

    torch.manual_seed(0)
    cfg = HLRTConfig(vocab_size=1024, d_model=256, tier1_num_layers=2, tier1_num_heads=2, tier1_d_ff=512,
                     gate1_chunk_size=16, num_latent_vectors=4, latent_pool_num_heads=2, tier2_d_model=256,
                     tier2_num_layers=1, tier2_num_heads=2, tier2_d_ff=512, tier3_d_model=256, tier3_num_layers=1,
                     tier3_num_heads=2, tier3_d_ff=512)
    model = HLRT(cfg).cuda().to(torch.bfloat16)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    ids = torch.randint(0, 1024, (2, 256), device="cuda")
    losses = []
    with linear_precision("nvfp4"):
        for _ in range(6):
            out = model(ids)
            loss = torch.nn.functional.cross_entropy(out["logits"][:, :-1].float().reshape(-1, 1024), ids[:, 1:].reshape(-1))
            loss.backward()
            opt.step()
            opt.zero_grad()
            losses.append(float(loss))
    assert all(l == l for l in losses) and losses[-1] < losses[0]


def test_nvfp4_unswizzle_inverts_swizzle():
    from llm_research_b200.ops.quant import nvfp4_swizzle_scales, nvfp4_unswizzle_scales

    s = torch.arange(256 * 32, dtype=torch.int64).remainder(127).to(torch.uint8).view(256, 32)
    back = nvfp4_unswizzle_scales(nvfp4_swizzle_scales(s), 256).view(torch.uint8)
    assert torch.equal(back, s)


def test_nvfp4_quantize_dual_cpu_oracle_shapes():
    from llm_research_b200.ops.quant import nvfp4_quantize_dual

    x = torch.randn(256, 384)
    row, col, st = nvfp4_quantize_dual(x)
    assert row.shape == (256, 384) and col.shape == (384, 256)
    torch.testing.assert_close(col.dequantize(), nvfp4_quantize_dual(x.t().contiguous(), colwise=False)[0].dequantize())


@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(128, 128), (256, 640), (1024, 4096)])
def test_nvfp4_quantize_dual_matches_rowwise_quantizer(M, K):
    """Row-wise output == the one-block-per-thread quantiser of x, transposed output ==
    the same quantiser of x^T (bit-exact, round to nearest); scales land in atom layout."""
    from llm_research_b200.ops.quant import nvfp4_quantize, nvfp4_quantize_dual, nvfp4_swizzle_scales

    torch.manual_seed(1)
    x = (torch.randn(M, K, device="cuda") * torch.rand(M, 1, device="cuda") * 4).to(torch.bfloat16)
    row, col, st = nvfp4_quantize_dual(x)
    p, s, st1 = nvfp4_quantize(x)
    pt, sT, st2 = nvfp4_quantize(x.t().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(row.packed, p) and torch.equal(row.atoms, nvfp4_swizzle_scales(s))
    assert torch.equal(col.packed, pt) and torch.equal(col.atoms, nvfp4_swizzle_scales(sT))
    assert float(st) == float(st1) == float(st2)


@pytest.mark.gpu
def test_nvfp4_quantize_dual_stochastic_is_unbiased():
    from llm_research_b200.ops.quant import nvfp4_quantize_dual

    torch.manual_seed(2)
    x = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
    acc_r = torch.zeros(256, 256, device="cuda")
    acc_c = torch.zeros(256, 256, device="cuda")
    n = 64
    for i in range(n):
        row, col, _ = nvfp4_quantize_dual(x, stochastic=True, seed=100 + i)
        acc_r += row.dequantize()
        acc_c += col.dequantize().t()
    ref = x.float()
    for acc in (acc_r, acc_c):
        bias = ((acc / n - ref).norm() / ref.norm()).item()
        assert bias < 0.035, bias


@pytest.mark.gpu
def test_nvfp4_stochastic_rounding_picks_a_neighbour_with_the_right_odds():
    """Stochastic rounding onto the E2M1 grid: values with known neighbours
    (one 16-element block with amax 6 so the block scale is 1) round only to
    those two grid points, with the probability of the upper one equal to the
    distance from the lower one over the spacing; element order in the packed
    bytes checked through the grid points themselves."""
    from llm_research_b200.ops.quant import nvfp4_quantize_dual

    base = torch.tensor([6.0, 0.3, -0.3, 1.25, 2.5, 3.5, 5.0, -4.5, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, -6.0])
    x = base.repeat(128, 8).to("cuda").to(torch.bfloat16)  # (128, 128): every block holds the 16 values
    lo = torch.tensor([6.0, 0.0, -0.5, 1.0, 2.0, 3.0, 4.0, -6.0, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, -6.0])
    hi = torch.tensor([6.0, 0.5, 0.0, 1.5, 3.0, 4.0, 6.0, -4.0, 0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, -6.0])
    ups = torch.zeros(16)
    n = 32
    for i in range(n):
        row, _, _ = nvfp4_quantize_dual(x, stochastic=True, seed=7 + i)
        q = row.dequantize().float().cpu().view(128, 8, 16)  # block scale x tensor scale = 1 up to rounding
        is_lo = torch.isclose(q, lo.expand_as(q), rtol=1e-5, atol=1e-6)
        is_hi = torch.isclose(q, hi.expand_as(q), rtol=1e-5, atol=1e-6)
        ok = is_lo | is_hi
        assert bool(ok.all()), q[~ok][:8]
        ups += is_hi.float().mean(dim=(0, 1))
    p_up = ups / n
    want = torch.where(hi != lo, (base - lo) / (hi - lo), torch.ones(16))
    assert torch.allclose(p_up, want, atol=0.03), (p_up, want)
