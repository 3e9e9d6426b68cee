"""CTA-pair tcgen05 GEMM (cta_group::2, 256 x 256 tiles) in every operand layout
against fp32 PyTorch: ragged M / N / K (tile and stage remainders, a pair whose
second CTA's rows lie wholly past M), bf16 / fp16 inputs, bf16 / fp16 / fp32
outputs and fp32 accumulation; then the three GEMMs of a linear layer."""

import pytest
import torch


def _ref(A, B, a_mn, b_mn):
    a = A.float().t() if a_mn else A.float()
    b = B.float() if b_mn else B.float().t()
    return a @ b


def _operands(M, N, K, a_mn, b_mn, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(*((K, M) if a_mn else (M, K)), device="cuda", generator=g).to(dtype)
    B = torch.randn(*((K, N) if b_mn else (N, K)), device="cuda", generator=g).to(dtype)
    return A, B


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (264, 520, 200), (1024, 768, 1024), (96, 40, 8)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_pair_layouts_bf16(M, N, K, a_mn, b_mn):
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    A, B = _operands(M, N, K, a_mn, b_mn, torch.bfloat16)
    C = gemm(A, B, a_mn, b_mn, alpha=0.5)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    ref = 0.5 * _ref(A, B, a_mn, b_mn)
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_gemm_pair_fp16_inputs_and_outputs(out_dtype):
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    A, B = _operands(520, 392, 328, False, True, torch.float16, seed=3)
    C = gemm(A, B, False, True, out_dtype=out_dtype)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    ref = _ref(A, B, False, True)
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 2e-3 if out_dtype == torch.float32 else 1e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn,b_mn", [(True, True), (False, False)])
def test_gemm_pair_accumulates_into_fp32(a_mn, b_mn):
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    A, B = _operands(384, 1000, 520, a_mn, b_mn, torch.bfloat16, seed=5)
    C0 = torch.randn(384, 1000, device="cuda")
    C = C0.clone()
    gemm(A, B, a_mn, b_mn, out=C, accumulate=True, alpha=2.0)
    gemm(A, B, a_mn, b_mn, out=C, accumulate=True, alpha=-1.0)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    ref = C0 + _ref(A, B, a_mn, b_mn)
    torch.testing.assert_close(C, ref, atol=2e-2, rtol=1e-3)


@pytest.mark.gpu
def test_gemm_pair_strided_operands_and_output():
    """Row pitches larger than the row (views into wider buffers)."""
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    g = torch.Generator(device="cuda").manual_seed(7)
    Abuf = torch.randn(300, 264, device="cuda", generator=g).bfloat16()
    Bbuf = torch.randn(520, 264, device="cuda", generator=g).bfloat16()
    A, B = Abuf[:, :200], Bbuf[:, :200]  # (300, 200) and (520, 200), pitch 264
    Cbuf = torch.zeros(300, 640, device="cuda", dtype=torch.bfloat16)
    C = Cbuf[:, 8:528]
    gemm(A, B, out=C)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    ref = A.float() @ B.float().t()
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err
    assert Cbuf[:, :8].abs().sum().item() == 0 and Cbuf[:, 528:].abs().sum().item() == 0


@pytest.mark.gpu
def test_linear_gemms_match_fp32():
    """forward x W^T, dgrad dY W and wgrad dY^T X at a small training shape."""
    from llm_research_b200.ops.gemm import gemm_pair_error, linear_dgrad, linear_fwd, linear_wgrad

    g = torch.Generator(device="cuda").manual_seed(11)
    T, K, N = 2048, 512, 1536
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    dy = torch.randn(T, N, device="cuda", generator=g).bfloat16()
    y, dx, dw = linear_fwd(x, w), linear_dgrad(dy, w), linear_wgrad(dy, x)
    acc = torch.zeros(N, K, device="cuda")
    linear_wgrad(dy, x, out=acc, accumulate=True)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    for got, ref in ((y, x.float() @ w.float().t()), (dx, dy.float() @ w.float()), (dw, dy.float().t() @ x.float()),
                     (acc, dy.float().t() @ x.float())):
        err = ((got.float() - ref).norm() / ref.norm()).item()
        assert err < 1e-2, err


@pytest.mark.gpu
def test_engine_direct_wgrad_accumulation_matches_returned_grads():
    """The sharding engine's fp32 gradient buffers after one bf16 micro-step: wgrad
    accumulated by the pair kernel straight into them equals dW returned through
    autograd and added by the engine, and both track an fp32 model."""
    import copy

    from genesis.model.hlrt import HLRT
    from llm_research_b200.models.presets import build_hlrt_config
    from llm_research_b200.ops.linear import set_direct_grad_accumulation
    from llm_research_b200.parallel.fsdp import FlatShardEngine

    cfg = build_hlrt_config("toy")
    torch.manual_seed(0)
    base = HLRT(cfg).cuda()
    with torch.no_grad():  # no escalation: gate scores near 0.5 would flip between bf16 and fp32
        base.gate1.gate_mlp[2].bias.fill_(-100.0)
    ids = torch.randint(0, cfg.vocab_size, (2, 128), device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))

    def grads(direct):
        set_direct_grad_accumulation(direct)
        try:
            eng = FlatShardEngine(copy.deepcopy(base), compute_dtype=torch.bfloat16)
            out = eng(ids)
            loss = torch.nn.functional.cross_entropy(out["logits"].float().flatten(0, 1), ids.flatten())
            (loss + out["aux_loss"]).backward()
            torch.cuda.synchronize()
            return {info.name: eng.units[info.unit].grad_acc[info.offset: info.offset + info.numel].clone()
                    for info in eng.params}
        finally:
            set_direct_grad_accumulation(True)

    direct, returned = grads(True), grads(False)
    ref_model = copy.deepcopy(base).float().cpu()  # fp32 oracle on the host
    out = ref_model(ids.cpu())
    (torch.nn.functional.cross_entropy(out["logits"].flatten(0, 1), ids.cpu().flatten()) + out["aux_loss"]).backward()
    ref = {n: p.grad.reshape(-1).cuda() for n, p in ref_model.named_parameters() if p.grad is not None}
    checked = 0
    for name, g in direct.items():
        r = returned[name]
        if r.norm() == 0:
            continue
        assert ((g - r).norm() / r.norm()).item() < 1e-2, name
        if name in ref:
            assert ((g - ref[name]).norm() / (ref[name].norm() + 1e-12)).item() < 5e-2, name
        checked += 1
    assert checked > 10


@pytest.mark.gpu
def test_gemm_pair_split_k_accumulation():
    """Few output tiles and a long K: the accumulating GEMM splits K over several
    CTA pairs whose partial sums meet in C through TMA reduce-adds."""
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    A, B = _operands(512, 512, 8192, True, True, torch.bfloat16, seed=9)
    C0 = torch.randn(512, 512, device="cuda")
    C = C0.clone()
    gemm(A, B, True, True, out=C, accumulate=True, alpha=0.25)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    ref = C0 + 0.25 * _ref(A, B, True, True)
    torch.testing.assert_close(C, ref, atol=5e-2, rtol=1e-3)


@pytest.mark.gpu
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_pair_unaligned_output_takes_direct_stores(out_dtype):
    """An output whose base is not 16-byte aligned cannot be a TMA target: the
    epilogue stores from registers instead."""
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    A, B = _operands(300, 264, 136, False, False, torch.bfloat16, seed=13)
    Cbuf = torch.zeros(300, 272, device="cuda", dtype=out_dtype)
    C = Cbuf[:, 1:265]
    gemm(A, B, out=C)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    ref = _ref(A, B, False, False)
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err
    assert Cbuf[:, 0].abs().sum().item() == 0 and Cbuf[:, 265:].abs().sum().item() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn,b_mn,acc", [(False, False, False), (False, True, False), (True, True, True)])
def test_gemm_pair_batched(a_mn, b_mn, acc):
    """A leading batch dimension: every entry is its own GEMM (grouped experts of
    equal shape), in one launch; ragged M / N per entry."""
    from llm_research_b200.ops.gemm import gemm, gemm_pair_error

    g = torch.Generator(device="cuda").manual_seed(17)
    E, M, N, K = 3, 200, 392, 264
    A = torch.randn(E, *((K, M) if a_mn else (M, K)), device="cuda", generator=g).bfloat16()
    B = torch.randn(E, *((K, N) if b_mn else (N, K)), device="cuda", generator=g).bfloat16()
    ref = torch.stack([_ref(A[e], B[e], a_mn, b_mn) for e in range(E)])
    if acc:
        C0 = torch.randn(E, M, N, device="cuda", generator=g)
        C = C0.clone()
        gemm(A, B, a_mn, b_mn, out=C, accumulate=True)
        ref = ref + C0
    else:
        C = gemm(A, B, a_mn, b_mn)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err


@pytest.mark.gpu
def test_grouped_swiglu_experts_match_fp32():
    """Grouped SwiGLU experts (forward and all gradients) against fp32 autograd."""
    from llm_research_b200.ops.gemm import gemm_pair_error
    from llm_research_b200.ops.linear import grouped_swiglu

    g = torch.Generator(device="cuda").manual_seed(19)
    E, R, d, F = 4, 136, 256, 384
    x = (torch.randn(E, R, d, device="cuda", generator=g)).bfloat16().requires_grad_()
    wug = (torch.randn(E, 2 * F, d, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    wd = (torch.randn(E, d, F, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    dy = torch.randn(E, R, d, device="cuda", generator=g).bfloat16()
    y = grouped_swiglu(x, wug, wd)
    y.backward(dy)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    xf, wugf, wdf = (t.detach().float().requires_grad_() for t in (x, wug, wd))
    gu = torch.bmm(xf, wugf.transpose(1, 2))
    u, gt = gu.chunk(2, dim=-1)
    yf = torch.bmm(torch.nn.functional.silu(gt) * u, wdf.transpose(1, 2))
    yf.backward(dy.float())
    for name, got, ref in (("y", y, yf), ("dx", x.grad, xf.grad), ("dwug", wug.grad, wugf.grad), ("dwd", wd.grad, wdf.grad)):
        err = ((got.float() - ref).norm() / ref.norm()).item()
        assert err < 2e-2, (name, err)


@pytest.mark.gpu
def test_swiglu_up_projection_matches_two_kernel_path():
    """One launch for [x W1^T | x Wg^T] and silu(g) * u, forward and backward,
    against the unfused GEMM + SwiGLU kernel and an fp32 oracle; ragged F and rows."""
    from llm_research_b200.ops.activation import swiglu
    from llm_research_b200.ops.gemm import gemm_pair_error
    from llm_research_b200.ops.linear import cat_rows, linear_bf16, swiglu_up

    g = torch.Generator(device="cuda").manual_seed(23)
    T, K, F = 1000, 512, 392
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16().requires_grad_()
    wbuf = (torch.randn(2 * F, K, device="cuda", generator=g) * 0.05).bfloat16()
    w1 = wbuf[:F].clone().requires_grad_()
    wg = wbuf[F:].clone().requires_grad_()
    dh = torch.randn(T, F, device="cuda", generator=g).bfloat16()
    h = swiglu_up(x, w1, wg)
    h.backward(dh)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    x2, w12, wg2 = (t.detach().clone().requires_grad_() for t in (x, w1, wg))
    h2 = swiglu(linear_bf16(x2, torch.cat([w12, wg2], 0)))
    h2.backward(dh)
    torch.testing.assert_close(h, h2, atol=2e-2, rtol=2e-2)
    xf, w1f, wgf = (t.detach().float().requires_grad_() for t in (x, w1, wg))
    hf = torch.nn.functional.silu(xf @ wgf.t()) * (xf @ w1f.t())
    hf.backward(dh.float())
    for name, got, ref in (("h", h, hf), ("dx", x.grad, xf.grad), ("dw1", w1.grad, w1f.grad), ("dwg", wg.grad, wgf.grad)):
        err = ((got.float() - ref).norm() / ref.norm()).item()
        assert err < 2e-2, (name, err)


@pytest.mark.gpu
@pytest.mark.parametrize("H,Hkv,offset", [(4, 4, 0), (8, 2, 5)])
def test_qkv_rope_epilogue_matches_separate_rotation(H, Hkv, offset):
    """QKV projection with RoPE in the epilogue against the GEMM followed by the
    rotation kernel, forward and backward (GQA, a position offset, ragged rows)."""
    from genesis.model.rotary import RotaryEmbedding
    from llm_research_b200 import ops
    from llm_research_b200.ops.gemm import gemm_pair_error
    from llm_research_b200.ops.linear import linear_bf16, qkv_rope

    g = torch.Generator(device="cuda").manual_seed(29)
    B, S, d, D = 2, 300, 256, 128
    N = (H + 2 * Hkv) * D
    rot = RotaryEmbedding(dim=D, max_seq_len=1024).cuda()
    cos, sin = rot(offset + S)
    x = torch.randn(B, S, d, device="cuda", generator=g).bfloat16().requires_grad_()
    w = (torch.randn(N, d, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    q, k, v = qkv_rope(x, w, cos, sin, H, Hkv, D, offset)
    x2, w2 = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    q2, k2, v2 = ops.rope_qkv(linear_bf16(x2, w2), cos, sin, H, Hkv, D, offset)
    for a, b in ((q, q2), (k, k2), (v, v2)):
        torch.testing.assert_close(a.float(), b.float(), atol=2e-2, rtol=2e-2)
    gq, gk, gv = (torch.randn(t.shape, device="cuda", generator=g).bfloat16() for t in (q, k, v))
    torch.autograd.backward((q, k, v), (gq, gk, gv))
    torch.autograd.backward((q2, k2, v2), (gq, gk, gv))
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    for name, a, b in (("dx", x.grad, x2.grad), ("dw", w.grad, w2.grad)):
        err = ((a.float() - b.float()).norm() / b.float().norm()).item()
        assert err < 1e-2, (name, err)


@pytest.mark.gpu
@pytest.mark.parametrize("batch,M,N,K", [(None, 264, 520, 200), (3, 512, 768, 256), (8, 256, 704, 256), (None, 96, 40, 64)])
@pytest.mark.parametrize("b_mn", [False, True])
def test_gemm_pair_axpby(batch, M, N, K, b_mn):
    """C = alpha A op(B)^T + beta D (the Newton-Schulz / residual epilogue, D staged
    by TMA two chunks ahead) against fp32, 2-D and batched, ragged tiles."""
    from llm_research_b200._ext import native
    from llm_research_b200.ops.gemm import gemm_pair_error

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    lead = () if batch is None else (batch,)
    A = torch.randn(*lead, M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(*lead, *((K, N) if b_mn else (N, K)), device="cuda", generator=g).bfloat16()
    D = torch.randn(*lead, M, N, device="cuda", generator=g).bfloat16()
    C = torch.empty(*lead, M, N, device="cuda", dtype=torch.bfloat16)
    native().gemm_pair_axpby(A, B, b_mn, C, D, 0.75, -1.5)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    Bf = B.float() if b_mn else B.float().transpose(-1, -2)
    ref = 0.75 * (A.float() @ Bf) - 1.5 * D.float()
    err = ((C.float() - ref).norm() / ref.norm()).item()
    assert err < 1e-2, err


@pytest.mark.gpu
def test_project_residual_epilogue_matches_separate_add():
    """r + x W^T with the residual in the GEMM epilogue: forward and the gradients
    of x, W and r against fp32 autograd; ragged rows."""
    from llm_research_b200.ops.gemm import gemm_pair_error
    from llm_research_b200.ops.linear import project_residual

    g = torch.Generator(device="cuda").manual_seed(31)
    T, K, N = 1000, 768, 520
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16().requires_grad_()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    r = torch.randn(T, N, device="cuda", generator=g).bfloat16().requires_grad_()
    dy = torch.randn(T, N, device="cuda", generator=g).bfloat16()
    y = project_residual(x, w, r)
    y.backward(dy)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    xf, wf, rf = (t.detach().float().requires_grad_() for t in (x, w, r))
    yf = rf + xf @ wf.t()
    yf.backward(dy.float())
    for name, got, ref in (("y", y, yf), ("dx", x.grad, xf.grad), ("dw", w.grad, wf.grad), ("dr", r.grad, rf.grad)):
        err = ((got.float() - ref).norm() / ref.norm()).item()
        assert err < 1e-2, (name, err)


@pytest.mark.gpu
@pytest.mark.parametrize("with_residual", [False, True])
def test_swiglu_ffn_fused_node_matches_fp32(with_residual):
    """The whole SwiGLU FFN as one node (up/gate + SwiGLU epilogue, down GEMM with
    the residual epilogue, down dgrad with the SwiGLU-backward epilogue) against
    fp32 autograd: output and the gradients of x, W1, Wg, W2 and the residual;
    ragged F and rows."""
    from llm_research_b200.ops.gemm import gemm_pair_error
    from llm_research_b200.ops.linear import swiglu_ffn

    g = torch.Generator(device="cuda").manual_seed(37)
    T, d, F = 1000, 512, 392
    x = torch.randn(T, d, device="cuda", generator=g).bfloat16().requires_grad_()
    w1 = (torch.randn(F, d, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    wg = (torch.randn(F, d, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    w2 = (torch.randn(d, F, device="cuda", generator=g) * 0.05).bfloat16().requires_grad_()
    r = torch.randn(T, d, device="cuda", generator=g).bfloat16().requires_grad_() if with_residual else None
    dy = torch.randn(T, d, device="cuda", generator=g).bfloat16()
    y = swiglu_ffn(x, w1, wg, w2, r)
    assert y is not None
    y.backward(dy)
    torch.cuda.synchronize()
    assert gemm_pair_error(0) == 0
    leaves = [x, w1, wg, w2] + ([r] if with_residual else [])
    fl = [t.detach().float().requires_grad_() for t in leaves]
    xf, w1f, wgf, w2f = fl[:4]
    yf = (torch.nn.functional.silu(xf @ wgf.t()) * (xf @ w1f.t())) @ w2f.t()
    if with_residual:
        yf = yf + fl[4]
    yf.backward(dy.float())
    err = ((y.float() - yf).norm() / yf.norm()).item()
    assert err < 2e-2, ("y", err)
    for name, got, ref in zip(["dx", "dw1", "dwg", "dw2", "dr"], leaves, fl):
        e = ((got.grad.float() - ref.grad).norm() / ref.grad.norm()).item()
        assert e < 3e-2, (name, e)
