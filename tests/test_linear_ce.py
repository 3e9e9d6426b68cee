"""Chunked linear + cross-entropy (the head without full logits) against the
logits path: the loss and every gradient agree."""

import torch
import torch.nn.functional as F


def test_linear_cross_entropy_matches_full_logits():
    from llm_research_b200.ops.loss import linear_cross_entropy

    torch.manual_seed(0)
    h = torch.randn(100, 32, requires_grad=True)
    w = torch.randn(50, 32, requires_grad=True)
    t = torch.randint(0, 50, (100,))
    t[::7] = -100
    loss = linear_cross_entropy(h, w, t, chunk=17)
    (2.0 * loss).backward()
    h2, w2 = h.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    ref = F.cross_entropy(h2 @ w2.t(), t, ignore_index=-100)
    (2.0 * ref).backward()
    torch.testing.assert_close(loss, ref)
    torch.testing.assert_close(h.grad, h2.grad)
    torch.testing.assert_close(w.grad, w2.grad)


def test_hlrt_ntp_with_fused_head_matches_logits_path():
    from genesis.model.hlrt import HLRT
    from genesis.training.train_phase1_bootstrap import ntp_objective
    from llm_research_b200.models.presets import build_hlrt_config

    cfg = build_hlrt_config("toy")
    ids = torch.randint(0, cfg.vocab_size, (2, 48), generator=torch.Generator().manual_seed(1))
    grads = []
    for fused in (False, True):
        torch.manual_seed(0)
        m = HLRT(cfg)
        loss = ntp_objective({"hlrt": m}, None, {"input_ids": ids, "fused_lm_loss": fused})
        loss.backward()
        grads.append((float(loss), {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}))
    assert abs(grads[0][0] - grads[1][0]) < 1e-5
    for n, g in grads[0][1].items():
        torch.testing.assert_close(grads[1][1][n], g, atol=1e-5, rtol=1e-4, msg=n)
