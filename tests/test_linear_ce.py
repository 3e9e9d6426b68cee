"""Chunked linear + cross-entropy (the head without full logits) against the
logits path: the loss and every gradient agree."""

import pytest
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


@pytest.mark.gpu
@pytest.mark.parametrize("ignore", [-100, -1])
def test_ce_bwd_vocab_shard_kernel_matches_fp32(ignore):
    """Gradient of one vocabulary shard's logits against the fp32 softmax of the
    full row; rows owned by another shard carry the marker the op assigns them
    (-1, or -2 when ignore_index is -1)."""
    from llm_research_b200._ext import native

    g = torch.Generator().manual_seed(5)
    R, V, v0, v1 = 300, 1000, 400, 720
    full = torch.randn(R, V, generator=g) * 3
    t = torch.randint(0, V, (R,), generator=g)
    t[::9] = ignore
    lse = torch.logsumexp(full, dim=-1)
    loc = full[:, v0:v1].to(torch.bfloat16)
    owned = (t >= v0) & (t < v1)
    other = -2 if ignore == -1 else -1
    t_loc = torch.where(owned, t - v0, torch.where(t != ignore, torch.full_like(t, other), t))
    scale = torch.tensor([0.25])
    got = native().ce_bwd_vocab_shard(loc.cuda(), t_loc.cuda(), lse.cuda(), scale.cuda(), ignore).float().cpu()
    p = torch.exp(loc.float() - lse[:, None])
    rows = torch.arange(R)[owned]
    p[rows, t_loc[owned]] -= 1.0
    ref = p * ((t != ignore).float() * 0.25)[:, None]
    torch.testing.assert_close(got, ref, atol=2e-3, rtol=2e-2)


@pytest.mark.gpu
def test_vocab_parallel_linear_cross_entropy_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from tests.dist_utils import run_ranks

    for res in run_ranks(_vocab_ce_gpu_case, 2, backend="nccl"):
        for r, got in zip(res["full"], res["vp"]):
            torch.testing.assert_close(got.float(), r.float(), atol=2e-2, rtol=2e-2)


def _vocab_ce_gpu_case(rank, world):
    import torch.distributed as dist

    from llm_research_b200.ops.loss import linear_cross_entropy, vocab_parallel_linear_cross_entropy

    dev = torch.device("cuda", rank)
    g = torch.Generator().manual_seed(7)
    h = (torch.randn(1024, 256, generator=g)).to(dev, torch.bfloat16)
    w = (torch.randn(4000, 256, generator=g) * 0.05).to(dev, torch.bfloat16)
    t = torch.randint(0, 4000, (1024,), generator=g).to(dev)
    t[::11] = -100
    out = {}
    for name, fn in (("full", lambda a, b: linear_cross_entropy(a, b, t, chunk=512)),
                     ("vp", lambda a, b: vocab_parallel_linear_cross_entropy(a, b, t, dist.group.WORLD, chunk=512))):
        a, b = h.clone().requires_grad_(), w.clone().requires_grad_()
        loss = fn(a, b)
        loss.backward()
        out[name] = (loss.detach().cpu(), a.grad.cpu(), b.grad.cpu())
    return out


@pytest.mark.gpu
def test_vocab_parallel_linear_cross_entropy_one_rank_gpu():
    """The GPU path of the vocabulary-parallel op (NCCL collectives, shard kernel)
    on a one-rank group equals the plain chunked op."""
    from tests.dist_utils import run_ranks

    for res in run_ranks(_vocab_ce_gpu_case, 1, backend="nccl"):
        for r, got in zip(res["full"], res["vp"]):
            torch.testing.assert_close(got.float(), r.float(), atol=2e-2, rtol=2e-2)
