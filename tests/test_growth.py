"""HLRT growth surgery: widen, deepen and dense-to-MoE each leave the model's
output unchanged at the moment of growth, update the config, and the grown
model keeps training with the rebuilt optimizer (carried-over state for the
parameters that survived)."""

import pytest
import torch

from genesis.model.growth import HLRTGrowthController


def _model():
    from genesis.model.hlrt import HLRT
    from llm_research_b200.models.presets import build_hlrt_config

    cfg = build_hlrt_config("toy")
    torch.manual_seed(0)
    m = HLRT(cfg)
    m.eval()
    return m


def _logits(m, ids):
    with torch.no_grad():
        return m(ids)["logits"]


@pytest.mark.parametrize("kind,kwargs", [
    ("widen", {"factor": 1.5}),
    ("deepen", {"num_layers": 2, "position": "end"}),
    ("deepen", {"num_layers": 1, "position": "start"}),
    ("deepen", {"num_layers": 1, "position": 1}),
    ("dense_to_moe", {"num_experts": 4, "top_k": 2}),
])
def test_growth_preserves_function(kind, kwargs):
    from olympus.optim import MuonAdamWHybrid

    m = _model()
    ids = torch.randint(0, m.config.vocab_size, (2, 64), generator=torch.Generator().manual_seed(1))
    before = _logits(m, ids)
    opt = MuonAdamWHybrid(m.parameters())
    gc = HLRTGrowthController(m, opt, schedule=[(3, kind, kwargs)])
    ev = gc.maybe_grow(3, 5.0)
    assert ev is not None and ev.event_type == kind and ev.new_param_count > ev.old_param_count
    after = _logits(gc.model, ids)
    torch.testing.assert_close(after, before, atol=1e-5, rtol=1e-5)
    cfg = gc.model.config
    if kind == "widen":
        assert all(b.ffn.d_ff == cfg.tier1_d_ff for b in gc.model.tier1.layers) and cfg.tier1_d_ff == 384
    elif kind == "deepen":
        assert cfg.tier1_num_layers == len(gc.model.tier1.layers) == 2 + kwargs["num_layers"]
    else:
        assert cfg.tier1_moe_num_experts == 4
    assert isinstance(gc.optimizer, MuonAdamWHybrid)


def test_grown_model_trains_and_keeps_optimizer_state():
    from olympus.optim import MuonAdamWHybrid

    m = _model()
    m.train()
    ids = torch.randint(0, m.config.vocab_size, (2, 64), generator=torch.Generator().manual_seed(2))
    opt = MuonAdamWHybrid(m.parameters(), lr_muon=0.02, lr_adamw=1e-3)

    def step(model, o):
        out = model(ids)
        loss = torch.nn.functional.cross_entropy(out["logits"][:, :-1].flatten(0, 1), ids[:, 1:].flatten())
        o.zero_grad()
        (loss + out["aux_loss"]).backward()
        o.step()
        return float(loss)

    step(m, opt)
    emb = m.embeddings.weight
    gc = HLRTGrowthController(m, opt, schedule=[(1, "deepen", {"num_layers": 1})])
    gc.maybe_grow(1, 5.0)
    assert gc.optimizer.state[emb]  # the embedding survived: its moments carried over
    losses = [step(gc.model, gc.optimizer) for _ in range(5)]
    assert all(l == l for l in losses) and losses[-1] < losses[0]
