"""sm_100a kernels against plain fp32 PyTorch statements of the same ops."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _native_loaded():
    from llm_research_b200._ext import native

    native()  # raise if the extension is missing: no silent fallback on a GPU box
    torch.manual_seed(0)


def _rms_ref(x, w, eps):
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return n.float() * w.float()


@pytest.mark.parametrize("d,rows", [(64, 37), (96, 37), (768, 37), (2048, 37), (4096, 37), (2048, 5000)])
@pytest.mark.parametrize("residual", [False, True])
def test_rmsnorm_fwd_bwd(d, rows, residual):
    """d a multiple of 256 up to 2048 takes the one-HBM-read backward (rows over
    several blocks and several rows per warp with 5000 rows)."""
    from llm_research_b200 import ops

    x = torch.randn(rows, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    r = torch.randn(rows, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(d, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    if residual:
        y, s = ops.rms_norm_residual(x, r, w, 1e-6)
        out = y.float().sum() + (s.float() * 0.5).sum()
    else:
        y = ops.rms_norm(x, w, 1e-6)
        out = y.float().sum()
    out.backward()
    xr = x.detach().float().clone().requires_grad_(True)
    rr = r.detach().float().clone().requires_grad_(True)
    wr = w.detach().float().clone().requires_grad_(True)
    src = xr + rr if residual else xr
    yr = src * torch.rsqrt(src.pow(2).mean(-1, keepdim=True) + 1e-6) * wr
    outr = yr.sum() + ((src * 0.5).sum() if residual else 0.0)
    outr.backward()
    torch.testing.assert_close(y.float(), yr.detach(), atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(w.grad.float(), wr.grad, atol=0.5 * max(1.0, rows / 37) ** 0.5, rtol=3e-2)
    if residual:
        torch.testing.assert_close(r.grad.float(), rr.grad, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("F_", [64, 5632, 100])
def test_swiglu(F_):
    from llm_research_b200 import ops

    gu = torch.randn(33, 2 * F_, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    h = ops.swiglu(gu)
    dh = torch.randn_like(h)
    h.backward(dh)
    ref = gu.detach().float().requires_grad_(True)
    u, g = ref.chunk(2, -1)
    hr = F.silu(g) * u
    hr.backward(dh.float())
    torch.testing.assert_close(h.float(), hr.detach(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(gu.grad.float(), ref.grad, atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("H,Hkv,D", [(4, 4, 64), (16, 16, 128), (8, 2, 128), (4, 1, 32)])
def test_rope_qkv(H, Hkv, D):
    from genesis.model.rotary import RotaryEmbedding
    from llm_research_b200 import ops
    from llm_research_b200.ops.rope import rope_qkv as rope_cpu

    B, S, off = 2, 50, 3
    rope = RotaryEmbedding(D, max_seq_len=128).cuda()
    cos, sin = rope(S + off)
    qkv = torch.randn(B, S, (H + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    q, k, v = ops.rope_qkv(qkv, cos, sin, H, Hkv, D, off)
    g = [torch.randn_like(t) for t in (q, k, v)]
    torch.autograd.backward((q, k, v), g)
    qr_in = qkv.detach().cpu().float().requires_grad_(True)
    qr, kr, vr = rope_cpu(qr_in, cos.cpu(), sin.cpu(), H, Hkv, D, off)
    torch.autograd.backward((qr, kr, vr), [t.cpu().float() for t in g])
    for a, b in zip((q, k, v), (qr, kr, vr)):
        torch.testing.assert_close(a.float().cpu(), b.detach(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(qkv.grad.float().cpu(), qr_in.grad, atol=3e-2, rtol=3e-2)


def _attn_ref(q, k, v, causal, scale):
    from llm_research_b200.ops.attention import _reference

    return _reference(q.float(), k.float(), v.float(), causal, scale)


@pytest.mark.parametrize("B,Sq,Skv,H,Hkv,D,causal", [
    (2, 128, 128, 4, 4, 64, True),
    (1, 200, 200, 8, 2, 128, True),
    (2, 77, 77, 4, 4, 32, False),
    (1, 1, 65, 4, 4, 64, True),       # decode-shaped query against a cache
    (1, 96, 96, 16, 16, 96, True),
    (1, 64, 64, 2, 1, 16, True),
])
def test_flash_attention(B, Sq, Skv, H, Hkv, D, causal):
    from llm_research_b200 import ops

    q = torch.randn(B, Sq, H, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, Skv, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, Skv, Hkv, D, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    scale = 1.0 / math.sqrt(D)
    o = ops.attention(q, k, v, causal=causal)
    do = torch.randn_like(o)
    o.backward(do)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    orf = _attn_ref(qr, kr, vr, causal, scale)
    orf.backward(do.float())
    torch.testing.assert_close(o.float(), orf.detach(), atol=2e-2, rtol=2e-2)
    for a, b in ((q, qr), (k, kr), (v, vr)):
        torch.testing.assert_close(a.grad.float(), b.grad, atol=5e-2, rtol=5e-2)


@pytest.mark.parametrize("V", [32000, 1000, 77])
def test_cross_entropy(V):
    from llm_research_b200 import ops

    logits = (3 * torch.randn(4, 33, V, device="cuda")).to(torch.bfloat16).requires_grad_(True)
    ids = torch.randint(0, V, (4, 33), device="cuda")
    loss = ops.loss.shifted_cross_entropy(logits, ids)
    loss.backward()
    ref_l = logits.detach().float().requires_grad_(True)
    lr = F.cross_entropy(ref_l[:, :-1].reshape(-1, V), ids[:, 1:].reshape(-1))
    lr.backward()
    torch.testing.assert_close(loss.float(), lr.detach(), atol=1e-3, rtol=1e-3)
    torch.testing.assert_close(logits.grad.float(), ref_l.grad, atol=2e-4, rtol=5e-2)


@pytest.mark.parametrize("E,k", [(16, 2), (4, 1), (64, 2), (128, 8)])
def test_softmax_topk(E, k):
    from llm_research_b200 import ops
    from llm_research_b200.ops.routing import _softmax_topk_ref

    logits = torch.randn(300, E, device="cuda", requires_grad=True)
    w, idx, p = ops.softmax_topk(logits, k)
    wr, idxr, pr = _softmax_topk_ref(logits.detach(), k)
    torch.testing.assert_close(p, pr, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(w, wr, atol=1e-5, rtol=1e-5)
    assert torch.equal(idx, idxr)
    gw = torch.randn_like(w)
    (w * gw).sum().backward()
    lr = logits.detach().clone().requires_grad_(True)
    wr2, _, _ = _softmax_topk_ref(lr, k)
    (wr2 * gw).sum().backward()
    torch.testing.assert_close(logits.grad, lr.grad, atol=1e-4, rtol=1e-4)


def test_chunk_pool_and_compaction():
    from llm_research_b200 import ops

    x = torch.randn(3, 128, 40, device="cuda")
    torch.testing.assert_close(ops.chunk_mean_pool(x, 32), x.view(3, 4, 32, 40).mean(2), atol=1e-5, rtol=1e-5)
    mask = torch.rand(5, 300, device="cuda") > 0.6
    ids, valid, n = ops.compact_chunks(mask)
    ids_c, valid_c, n_c = ops.compact_chunks(mask.cpu())
    assert n == n_c
    assert torch.equal(ids.cpu(), ids_c) and torch.equal(valid.cpu(), valid_c)


def test_muon_and_adamw_kernels_match_cpu():
    from llm_research_b200 import ops

    shapes = [(64, 64), (128, 32), (33, 70)]
    ps = [torch.randn(s, device="cuda") for s in shapes]
    gs = [torch.randn(s, device="cuda") for s in shapes]
    bs = [torch.randn(s, device="cuda") for s in shapes]
    pc, gc, bc = ([t.cpu().clone() for t in l] for l in (ps, gs, bs))
    outs, gn = ops.muon_prologue(ps, gs, bs, 0.02, 0.95, 0.1, out_dtype=torch.float32)
    outs_c, gn_c = ops.muon_prologue(pc, gc, bc, 0.02, 0.95, 0.1)
    for a, b in zip(outs, outs_c):
        torch.testing.assert_close(a.cpu(), b, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(gn.cpu(), gn_c, atol=1e-4, rtol=1e-5)
    ops.muon_epilogue(ps, outs, gn, 0.02)
    ops.muon_epilogue(pc, outs_c, gn_c, 0.02)
    for a, b in zip(ps, pc):
        torch.testing.assert_close(a.cpu(), b, atol=1e-5, rtol=1e-5)
    m = [torch.zeros_like(p) for p in ps]
    v = [torch.zeros_like(p) for p in ps]
    mc = [t.cpu() for t in m]
    vc = [t.cpu() for t in v]
    for step in (1, 2):
        ops.adamw_step(ps, gs, m, v, [step] * 3, 3e-4, 0.9, 0.999, 1e-8, 0.01)
        ops.adamw_step(pc, gc, mc, vc, [step] * 3, 3e-4, 0.9, 0.999, 1e-8, 0.01)
    for a, b in zip(ps, pc):
        torch.testing.assert_close(a.cpu(), b, atol=1e-5, rtol=1e-5)


def test_newton_schulz_orthogonalises():
    from llm_research_b200 import ops

    G = torch.randn(3, 256, 512, device="cuda")
    X = ops.newton_schulz(G, steps=5)
    eye = torch.eye(256, device="cuda")
    prod = X.float() @ X.float().transpose(1, 2)
    assert (prod - eye).abs().max().item() < 0.5
    ref = ops.newton_schulz(G.cpu(), steps=5)
    assert (X.float().cpu() - ref).abs().max().item() < 0.1


@pytest.mark.parametrize("G", [-1, 32, 100])
def test_int4_quant(G):
    from llm_research_b200 import ops

    x = torch.randn(20, 256, device="cuda")
    q, s = ops.int4_quantize(x, G)
    qc, sc = ops.int4_quantize(x.cpu(), G)
    torch.testing.assert_close(s.cpu(), sc, atol=1e-6, rtol=1e-6)
    assert (q.cpu().int() - qc.int()).abs().max().item() <= 1  # ties may round differently
    y = ops.int4_dequantize(q, s, G)
    yc = ops.int4_dequantize(q.cpu(), s.cpu(), G)
    torch.testing.assert_close(y.cpu(), yc, atol=1e-6, rtol=1e-6)


def test_nvfp4_quant_roundtrip():
    from llm_research_b200 import ops

    x = torch.randn(64, 256, device="cuda")
    pk, sb, st = ops.nvfp4_quantize(x)
    pkc, sbc, stc = ops.nvfp4_quantize(x.cpu())
    torch.testing.assert_close(st.cpu(), stc, atol=0, rtol=1e-6)
    assert torch.equal(sb.cpu().view(torch.uint8), sbc.view(torch.uint8))
    assert torch.equal(pk.cpu(), pkc)
    y = ops.nvfp4_dequantize(pk, sb, st)
    rel = (y - x).norm() / x.norm()
    assert rel.item() < 0.15


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1000, 700, 520), (4096, 6144, 2048), (300, 4000, 4096), (37, 96, 16)])
@pytest.mark.parametrize("out", [torch.bfloat16, torch.float32])
def test_tcgen05_gemm(M, N, K, out):
    from llm_research_b200.ops.gemm import matmul_tn, sm100_error

    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    c = matmul_tn(a, b, out_dtype=out)
    ref = a.float() @ b.float().t()
    torch.cuda.synchronize()
    assert sm100_error() == 0
    torch.testing.assert_close(c.float(), ref, atol=2e-2 * (K ** 0.5), rtol=2e-2)


def test_tcgen05_gemm_accumulate():
    from llm_research_b200.ops.gemm import matmul_tn_accumulate, sm100_error

    a = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
    b = torch.randn(384, 256, device="cuda").to(torch.bfloat16)
    c = torch.randn(512, 384, device="cuda")
    ref = c + 0.5 * (a.float() @ b.float().t())
    matmul_tn_accumulate(a, b, c, alpha=0.5)
    torch.cuda.synchronize()
    assert sm100_error() == 0
    torch.testing.assert_close(c, ref, atol=0.05, rtol=1e-2)


def test_exp2_fma_polynomial_against_exp2():
    """The FMA-pipe 2^x used for a quarter of the attention softmax's exponentials:
    relative error within its 8.6e-5 bound against CUDA's exp2 (torch.exp2) over
    the range a softmax sees, exact powers of two at integers, and +0 at -inf."""
    from llm_research_b200._ext import native

    x = torch.cat([torch.linspace(-126.0, 12.0, 2_000_001, device="cuda"),
                   torch.arange(-126, 13, device="cuda", dtype=torch.float32)])
    got = native().exp2_fma_eval(x).double()
    ref = torch.exp2(x).double()
    rel = ((got - ref).abs() / ref).max().item()
    assert rel < 1e-4, rel
    ints = torch.arange(-126, 13, device="cuda", dtype=torch.float32)
    assert torch.equal(native().exp2_fma_eval(ints), torch.exp2(ints))
    z = native().exp2_fma_eval(torch.tensor([float("-inf"), -127.0, -500.0], device="cuda"))
    assert torch.equal(z, torch.zeros(3, device="cuda"))
