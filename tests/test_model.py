"""GENESIS model family on CPU: shapes, causality, gating, MoE, checkpoint
names, and parity with the reference implementation (same seed -> same
weights and the same outputs)."""

import pytest
import torch

from genesis.model import HLRT, HLRTConfig
from genesis.model.moe import MoEFFN
from genesis.model.tier1_token_processor import Tier1TokenProcessor
from genesis.model.tier_gate import TierGate

from tests.reference_oracle import reference_root, run_reference

TINY = dict(
    vocab_size=256, d_model=64, tier1_num_layers=2, tier1_num_heads=4, tier1_d_ff=128,
    gate1_chunk_size=4, num_latent_vectors=2, latent_pool_num_heads=2,
    tier2_d_model=64, tier2_num_layers=1, tier2_num_heads=4, tier2_d_ff=128,
    tier3_d_model=64, tier3_num_layers=1, tier3_num_heads=4, tier3_d_ff=128, tier3_recurrence_steps=2,
)


def _model(seed=0, **over):
    torch.manual_seed(seed)
    return HLRT(HLRTConfig(**{**TINY, **over}))


def test_forward_shapes_and_aux():
    m = _model()
    ids = torch.randint(0, 256, (2, 32))
    out = m(ids, return_tier_activations=True)
    assert out["logits"].shape == (2, 32, 256)
    assert out["aux_loss"].dim() == 0
    assert "tier1" in out["tier_activations"] and "gate1_scores" in out["tier_activations"]


def test_tier1_causality():
    torch.manual_seed(0)
    t1 = Tier1TokenProcessor(num_layers=2, d_model=32, num_heads=4, d_ff=64)
    x = torch.randn(1, 16, 32)
    y1 = t1(x)
    x2 = x.clone()
    x2[:, 10:] = torch.randn(1, 6, 32)
    y2 = t1(x2)
    torch.testing.assert_close(y1[:, :10], y2[:, :10])
    assert not torch.allclose(y1[:, 10:], y2[:, 10:])


def test_tier_gate_soft_and_hard():
    g = TierGate(d_model=32, chunk_size=4)
    x = torch.randn(2, 18, 32)  # padded to 20 -> 5 chunks
    g.train()
    mask, scores = g(x)
    assert mask.dtype == torch.float32 and mask.shape == (2, 5)
    g.eval()
    mask, _ = g(x)
    assert mask.dtype == torch.bool
    assert g.load_balance_loss().dim() == 0


def test_moe_matches_masked_loop_and_capacity():
    torch.manual_seed(0)
    moe = MoEFFN(d_model=32, d_ff=64, num_experts=4, top_k=2)
    x = torch.randn(2, 10, 32)
    y = moe(x)
    w, idx, _ = moe.router(x.view(-1, 32))
    ref = torch.zeros(20, 32)
    for k in range(2):
        for e in range(4):
            msk = idx[:, k] == e
            if msk.any():
                ref[msk] += w[msk, k:k + 1] * moe.experts[e](x.view(-1, 32)[msk])
    torch.testing.assert_close(y.view(-1, 32), ref, atol=1e-5, rtol=1e-5)
    assert moe.load_balance_loss().item() > 0
    moe.enforce_capacity = True
    moe.capacity_factor = 0.25
    assert moe(x).shape == x.shape


def test_checkpoint_parameter_names():
    m = _model(tier2_moe_num_experts=2)
    names = set(dict(m.named_parameters()))
    for n in ("embeddings.embedding.weight", "tier1.layers.0.attn.q_proj.weight", "tier1.layers.0.ffn.w_gate.weight",
              "gate1.gate_mlp.0.weight", "gate1.gate_mlp.2.bias", "latent_pool.learned_queries",
              "latent_pool.norm.bias", "tier2.layers.0.ffn.router.gate.weight", "tier2.layers.0.ffn.experts.1.w2.weight",
              "tier2.final_norm.weight", "tier3.step_embedding", "tier3.input_proj.weight",
              "conditioning.tier3_alpha", "conditioning.plan_proj.weight", "output_norm.weight"):
        assert n in names, n
    sd = m.state_dict_with_state()
    assert "last_plan_vector" in sd["_olympus_state_tensors"]
    assert not any("cos_cached" in k for k in sd)


def test_cached_decode_matches_full_forward_tier1():
    from genesis.inference.kv_cache import KVCache

    m = _model()
    m.eval()
    ids = torch.randint(0, 256, (1, 12))
    with torch.no_grad():
        full = m.tier1(m.embeddings(ids))
        cache = KVCache(num_layers=2)
        m.tier1(m.embeddings(ids[:, :11]), kv_cache=cache)
        last = m.tier1(m.embeddings(ids[:, 11:]), kv_cache=cache, position_offset=11)
    torch.testing.assert_close(last[:, 0], full[:, 11], atol=1e-5, rtol=1e-5)


_REF_CODE = r"""
import torch
from genesis.model.hlrt import HLRT, HLRTConfig
def run(a):
    torch.manual_seed(a['seed'])
    m = HLRT(HLRTConfig(**a['cfg']))
    m.train(a['train'])
    out = m(a['ids'])
    loss = out['logits'].float().pow(2).mean() + out['aux_loss']
    loss.backward()
    grads = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
    return {'sd': {k: v.clone() for k, v in m.state_dict().items()}, 'logits': out['logits'].detach(),
            'aux': out['aux_loss'].detach(), 'grads': grads}
"""


@pytest.mark.skipif(reference_root() is None, reason="reference not installed")
@pytest.mark.parametrize("train", [True, False])
def test_parity_with_reference_hlrt(train):
    ids = torch.randint(0, 256, (2, 24), generator=torch.Generator().manual_seed(3))
    ref = run_reference(_REF_CODE, {"seed": 7, "cfg": TINY, "ids": ids, "train": train})
    m = _model(seed=7)
    m.train(train)
    sd = m.state_dict()
    assert set(sd) == set(ref["sd"])
    for k, v in ref["sd"].items():
        torch.testing.assert_close(sd[k], v, atol=0, rtol=0, msg=k)  # identical initialisation
    out = m(ids)
    torch.testing.assert_close(out["logits"].detach(), ref["logits"], atol=2e-4, rtol=2e-4)
    torch.testing.assert_close(out["aux_loss"].detach(), ref["aux"], atol=1e-5, rtol=1e-5)
    loss = out["logits"].float().pow(2).mean() + out["aux_loss"]
    loss.backward()
    for n, p in m.named_parameters():
        if n in ref["grads"]:
            torch.testing.assert_close(p.grad, ref["grads"][n], atol=1e-4, rtol=1e-3, msg=n)
