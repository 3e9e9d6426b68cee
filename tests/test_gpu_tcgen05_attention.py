"""tcgen05/TMEM flash-attention forward against fp32 PyTorch attention."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,Sq,Skv,H,Hkv,causal", [
    (1, 128, 128, 1, 1, True),
    (2, 300, 300, 4, 2, True),
    (1, 1, 200, 4, 4, True),
    (1, 1000, 1000, 8, 8, False),
    (1, 77, 300, 2, 1, True),
    (2, 2048, 2048, 4, 4, True),
])
def test_tcgen05_attention_forward(B, Sq, Skv, H, Hkv, causal):
    from llm_research_b200._ext import native
    from llm_research_b200.ops.attention import _reference

    torch.manual_seed(0)
    q = torch.randn(B, Sq, H, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, Skv, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, Skv, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    C = native()
    assert C.attn_sm100_supported(q, k, v)
    o, lse = C.attn_fwd_sm100(q, k, v, causal, scale)
    torch.cuda.synchronize()
    assert C.attn_sm100_error(0) == 0
    ref = _reference(q.float(), k.float(), v.float(), causal, scale)
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)
    o2, lse2 = C.attn_fwd(q, k, v, causal, scale)
    finite = torch.isfinite(lse2)
    torch.testing.assert_close(lse[finite], lse2[finite], atol=1e-3, rtol=1e-3)


def test_tcgen05_attention_strided_qkv_views():
    """q/k/v as views into one packed projection output (the model's layout)."""
    from llm_research_b200._ext import native
    from llm_research_b200.ops.attention import _reference

    B, S, H = 2, 256, 4
    qkv = torch.randn(B, S, 3 * H * 128, device="cuda", dtype=torch.bfloat16)
    q, k, v = qkv.view(B, S, 3 * H, 128).split(H, dim=2)
    o, _ = native().attn_fwd_sm100(q, k, v, True, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    ref = _reference(q.float(), k.float(), v.float(), True, 1 / math.sqrt(128))
    torch.testing.assert_close(o.float(), ref, atol=2e-2, rtol=2e-2)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("B,Sq,Skv,H,Hkv,causal", [
    (1, 128, 128, 1, 1, True),
    (2, 300, 300, 4, 2, True),
    (1, 77, 300, 2, 1, True),
    (1, 1000, 1000, 2, 2, False),
    (2, 1024, 1024, 8, 2, True),
])
def test_tcgen05_attention_backward(B, Sq, Skv, H, Hkv, causal):
    """tcgen05 backward vs fp32 autograd of the reference and vs the mma.sync backward."""
    from llm_research_b200._ext import native
    from llm_research_b200.ops.attention import _reference

    torch.manual_seed(1)
    q = torch.randn(B, Sq, H, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, Skv, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, Skv, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    dout = torch.randn(B, Sq, H, 128, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(128)
    C = native()
    o, lse = C.attn_fwd_sm100(q, k, v, causal, scale)
    dq, dk, dv = C.attn_bwd(dout, q, k, v, o, lse, causal, scale, True)
    torch.cuda.synchronize()
    assert C.attn_bwd_sm100_error(0) == 0
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    _reference(qf, kf, vf, causal, scale).backward(dout.float())
    for name, got, ref in (("dq", dq, qf.grad), ("dk", dk, kf.grad), ("dv", dv, vf.grad)):
        assert _rel(got, ref) < 2e-2, (name, _rel(got, ref))
    dq2, dk2, dv2 = C.attn_bwd(dout, q, k, v, o, lse, causal, scale, False)
    for name, got, ref in (("dq", dq, dq2), ("dk", dk, dk2), ("dv", dv, dv2)):
        assert _rel(got, ref) < 2e-2, (name, _rel(got, ref))
