"""PHMA memory read: fused tcgen05 similarity + streaming top-32, the value
gather and its backward, against the explicit fp32 similarity matrix."""

import pytest
import torch
import torch.nn.functional as F


def _bank(N, D, seed=0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    keys = F.normalize(torch.randn(N, D, generator=g), dim=-1).to(torch.bfloat16)
    values = (torch.randn(N, D, generator=g)).to(torch.bfloat16)
    return keys.to(device), values.to(device)


def test_bank_read_cpu_oracle_matches_semantic_memory_read():
    """The CPU path is the semantic-memory read: cosine top-k, softmax over the k sims."""
    from llm_research_b200.ops.memory import bank_read, topk_memory_read

    keys, values = _bank(512, 64)
    keys = F.normalize(keys.float(), dim=-1)
    q = torch.randn(10, 64)
    out, idx = bank_read(q, keys, values.float(), 8)
    ref = topk_memory_read(q, keys, values.float(), 8)
    torch.testing.assert_close(out.float(), ref, atol=1e-5, rtol=1e-5)


def test_memory_layer_trains_on_cpu():
    from genesis.model.hlrt import HLRT
    from llm_research_b200.models.presets import build_hlrt_config

    cfg = build_hlrt_config("toy")
    cfg.tier1_memory_every = 1
    cfg.memory_slots = 256
    cfg.memory_top_k = 4
    torch.manual_seed(0)
    m = HLRT(cfg)
    assert len(m.tier1.memory_layers) == cfg.tier1_num_layers
    sd = m.state_dict()
    assert sum(1 for k in sd if k.endswith("memory_bank.keys")) == 1  # the shared bank is saved once
    ids = torch.randint(0, cfg.vocab_size, (2, 32))
    out = m(ids)
    out["logits"].float().sum().backward()
    assert m.tier1.memory_layers["0"].query_proj.weight.grad is not None
    assert m.tier1.memory_layers["0"].query_proj.weight.grad.abs().sum() > 0


@pytest.mark.gpu
@pytest.mark.parametrize("T,N,D", [(128, 256, 64), (300, 5000, 128), (1024, 65536, 512)])
def test_memory_topk_candidates_select_the_best_slots(T, N, D):
    from llm_research_b200._ext import native

    keys, _ = _bank(N, D, device="cuda")
    q = F.normalize(torch.randn(T, D, device="cuda"), dim=-1).to(torch.bfloat16)
    cs, ci = native().memory_topk_candidates(q, keys, 0)
    torch.cuda.synchronize()
    assert native().memory_topk_error(0) == 0
    cand_s = cs.permute(1, 0, 2).reshape(T, -1)
    cand_i = ci.permute(1, 0, 2).reshape(T, -1)
    top, pos = cand_s.topk(32, dim=1)
    idx = cand_i.gather(1, pos).long()
    sim = q.float() @ keys.float().t()
    # returned scores are the similarities of the returned slots
    torch.testing.assert_close(top, sim.gather(1, idx), atol=2e-3, rtol=1e-3)
    # and they are the 32 best up to accumulation-order ties
    ref_top = sim.topk(32, dim=1).values
    assert (top[:, -1] >= ref_top[:, -1] - 2e-3).all()
    assert (top[:, 0] >= ref_top[:, 0] - 2e-3).all()
    assert (idx >= 0).all() and (idx < N).all()
    assert all(len(set(r.tolist())) == 32 for r in idx[:64])


@pytest.mark.gpu
def test_bank_read_forward_backward_matches_oracle():
    from llm_research_b200.ops.memory import bank_read

    T, N, D = 256, 8192, 256
    keys, values = _bank(N, D, seed=3, device="cuda")
    q = torch.randn(T, D, device="cuda", requires_grad=True)
    out, idx = bank_read(q, keys, values, 32)
    g = torch.randn(T, D, device="cuda")
    (out.float() * g).sum().backward()
    dq = q.grad.clone()
    # oracle on the same selection, in fp32
    q2 = q.detach().clone().requires_grad_()
    qn = F.normalize(q2, dim=-1)
    s = (qn.unsqueeze(1) * keys.float()[idx.long()]).sum(-1)
    w = F.softmax(s, dim=-1)
    ref = (w.unsqueeze(-1) * values.float()[idx.long()]).sum(1)
    (ref * g).sum().backward()
    assert ((out.float() - ref).norm() / ref.norm()).item() < 1e-2
    assert ((dq - q2.grad).norm() / q2.grad.norm()).item() < 2e-2
