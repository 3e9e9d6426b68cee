"""Olympus core runtime: StatefulModule/StateLink, MemoryBus, ComputeRouter,
TrainingOrchestrator (incl. the reference checkpoint layout), GrowthController."""

import os

import pytest
import torch
import torch.nn as nn

from olympus.core import (
    ComputeRouter, GrowthController, MemoryBus, ModelConfig, ObjectiveConfig, RoutePlan, StatefulModule, StateLink,
    TrainingContext, TrainingOrchestrator,
)


class Tiny(StatefulModule):
    def __init__(self, dim=16):
        super().__init__()
        self.linear = nn.Linear(dim, dim)
        self.register_state("hidden", torch.zeros(dim))
        self.register_memory("ctx", torch.zeros(dim))

    def forward(self, x):
        out = self.linear(x + self.link_state("hidden"))
        self.set_state("hidden", out.detach().mean(0) if out.dim() > 1 else out.detach())
        return out


# ---------------------------------------------------------------- stateful
def test_state_and_memory_registration():
    m = Tiny()
    assert m.state_names() == ["hidden"] and m.memory_names() == ["ctx"]
    with pytest.raises(ValueError, match="already registered"):
        m.register_state("hidden", torch.zeros(16))
    with pytest.raises(ValueError, match="already registered"):
        m.register_memory("ctx", torch.zeros(16))
    with pytest.raises(KeyError):
        m.get_state("nope")


def test_state_persists_and_updates():
    torch.manual_seed(0)
    m = Tiny()
    x = torch.randn(16)
    out = m(x)
    assert torch.allclose(m.get_state("hidden"), out.detach())
    s1 = m.get_state("hidden").clone()
    m(x)
    assert not torch.allclose(s1, m.get_state("hidden"))


def test_statelink_accumulates_gradients():
    m = Tiny()
    t = torch.ones(16, requires_grad=True)
    (StateLink.apply(t, m, "hidden") ** 2).sum().backward()
    g1 = m._state_grads["hidden"].clone()
    (StateLink.apply(t, m, "hidden") * 3).sum().backward()
    assert torch.allclose(m._state_grads["hidden"], g1 + 3)
    m.zero_state_grads()
    assert m._state_grads["hidden"] is None


def test_apply_state_grads_is_sgd():
    m = Tiny()
    m._state_grads["hidden"] = torch.ones(16)
    before = m.get_state("hidden").clone()
    m.apply_state_grads(lr=0.1)
    assert torch.allclose(m.get_state("hidden"), before - 0.1)
    assert m._state_grads["hidden"] is None


def test_state_dict_with_state_roundtrip_and_keys():
    m = Tiny()
    m(torch.randn(16))
    m.update_memory("ctx", torch.randn(16))
    sd = m.state_dict_with_state()
    for k in ("_olympus_state_tensors", "_olympus_state_meta", "_olympus_memory_tensors", "_olympus_memory_meta"):
        assert k in sd
    fresh = Tiny()
    fresh.load_state_dict_with_state(dict(sd))
    assert torch.allclose(fresh.get_state("hidden"), m.get_state("hidden"))
    assert torch.allclose(fresh.get_memory("ctx"), m.get_memory("ctx"))


def test_to_moves_state():
    m = Tiny().to(torch.float64)
    assert m.get_state("hidden").dtype == torch.float64
    assert m._state_tensors["hidden"].dtype == torch.float64


# ---------------------------------------------------------------- bus
def test_memory_bus_scopes_and_query():
    bus = MemoryBus()
    bus.write("a", torch.tensor([1.0, 0.0]), scope="step")
    bus.write("b", torch.tensor([0.0, 1.0]), scope="permanent")
    bus.write("c", torch.tensor([1.0, 1.0, 0.0]), scope="permanent")
    assert bus.read("a") is not None
    bus.step()
    assert bus.read("a") is None and bus.read("b", "permanent") is not None
    res = bus.query(torch.tensor([0.0, 1.0]), scope="permanent", top_k=2)
    assert res[0][0] == "b" and abs(res[0][2] - 1.0) < 1e-6
    with pytest.raises(ValueError):
        bus.write("x", torch.zeros(1), scope="bogus")
    v = bus.read("b", "permanent")
    v += 5
    assert bus.read("b", "permanent")[1] == 1.0  # copies out
    sd = bus.state_dict()
    assert set(sd) == {"permanent", "episode"}
    bus2 = MemoryBus()
    bus2.load_state_dict(sd)
    assert bus2.list_keys("permanent") == ["b", "c"]
    bus.clear_all()
    assert bus.list_keys("permanent") == []


# ---------------------------------------------------------------- router
@pytest.mark.parametrize("gate", ["linear", "mlp", "entropy"])
def test_compute_router(gate):
    torch.manual_seed(0)
    r = ComputeRouter(input_dim=32, num_experts=4, top_k=2, gate_type=gate)
    x = torch.randn(4, 8, 32, requires_grad=True)
    plan = r.plan(x)
    assert isinstance(plan, RoutePlan) and plan.expert_indices.shape == (32, 2) and plan.num_experts == 4
    assert torch.allclose(plan.expert_weights.sum(-1), torch.ones(32), atol=1e-5)
    experts = nn.ModuleList([nn.Linear(32, 32) for _ in range(4)])
    out = r.execute(x, experts)
    assert out.shape == x.shape
    out.sum().backward()
    assert x.grad is not None
    lb = r.load_balance_loss(plan)
    assert lb.dim() == 0 and (gate == "entropy" or lb.item() >= 0)
    stats = r.get_routing_stats()
    assert stats["total_tokens"] == 64 and len(stats["expert_utilization"]) == 4  # plan() + execute() both route
    with pytest.raises(ValueError):
        ComputeRouter(input_dim=8, num_experts=2, gate_type="bogus")


def test_router_execute_matches_masked_loop():
    torch.manual_seed(1)
    r = ComputeRouter(input_dim=16, num_experts=3, top_k=2)
    experts = nn.ModuleList([nn.Linear(16, 16) for _ in range(3)])
    x = torch.randn(40, 16)
    plan = r.plan(x)
    got = r.execute(x, experts, plan)
    ref = torch.zeros_like(x)
    for k in range(2):
        for e in range(3):
            msk = plan.expert_indices[:, k] == e
            if msk.any():
                ref[msk] += plan.expert_weights[msk, k:k + 1] * experts[e](x[msk])
    torch.testing.assert_close(got, ref, atol=1e-5, rtol=1e-5)


# ---------------------------------------------------------------- orchestrator
def _orch(accum=1):
    torch.manual_seed(0)
    model = Tiny(8)
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    o = TrainingOrchestrator(gradient_accumulation_steps=accum)
    o.add_model(ModelConfig("m", model, opt, enabled_phases=["bootstrap"]))
    o.add_objective(ObjectiveConfig("mse", lambda ms, ctx, b: (ms["m"](b) ** 2).mean()))
    return o, model


def test_orchestrator_accumulation_and_phases():
    o, model = _orch(accum=2)
    w0 = model.linear.weight.detach().clone()
    o.step(torch.randn(4, 8))
    assert torch.equal(w0, model.linear.weight) and o.global_step == 0
    out = o.step(torch.randn(4, 8))
    assert o.global_step == 1 and not torch.equal(w0, model.linear.weight)
    assert set(out) == {"mse", "total"} and isinstance(out["total"], float)
    with pytest.raises(ValueError):
        o.add_model(ModelConfig("m", model, torch.optim.SGD(model.parameters(), lr=0.1)))
    ctx = TrainingContext(gradient_accumulation_steps=4, current_accumulation_step=1)
    assert ctx.is_accumulating and ctx.tokens_seen == 0


def test_orchestrator_checkpoint_layout(tmp_path):
    o, model = _orch()
    o.memory_bus.write("k", torch.ones(3), scope="permanent")
    o.step(torch.randn(4, 8))
    p = str(tmp_path / "c.pt")
    o.save_checkpoint(p)
    ck = torch.load(p, weights_only=False)
    # the reference's keys, plus the generator states (an extension its loaders ignore)
    assert set(ck) == {"global_step", "epoch", "phase", "prev_loss", "memory_bus", "models", "optimizers", "schedulers",
                       "rng_state"}
    assert "_olympus_state_tensors" in ck["models"]["m"]
    o2, model2 = _orch()
    o2.load_checkpoint(p)
    assert o2.global_step == 1
    assert torch.equal(model2.linear.weight, model.linear.weight)
    assert torch.equal(o2.memory_bus.read("k", "permanent"), torch.ones(3))


# ---------------------------------------------------------------- growth
class _Grow(GrowthController):
    def _widen(self, model, factor=2.0, **kw):
        return nn.Linear(4, int(4 * factor))


def test_growth_controller_schedule_and_plateau():
    m = nn.Linear(4, 4)
    gc = _Grow(m, torch.optim.SGD(m.parameters(), lr=0.1), schedule=[(2, "widen", {"factor": 2.0})], patience=3)
    assert gc.maybe_grow(1, 1.0) is None
    ev = gc.maybe_grow(2, 1.0)
    assert ev.event_type == "widen" and ev.new_param_count > ev.old_param_count
    for s in range(3, 6):
        ev = gc.maybe_grow(s, 1.0)
    assert ev is not None and ev.metadata == {"factor": 1.5}
    # rebuilt as the same optimizer class with the old defaults
    assert len(gc.history) == 2 and type(gc.optimizer) is torch.optim.SGD and gc.optimizer.defaults["lr"] == 0.1
    with pytest.raises(NotImplementedError):
        GrowthController(m, torch.optim.SGD(m.parameters(), lr=0.1), schedule=[(0, "deepen", {})]).maybe_grow(0, 1.0)
    with pytest.raises(ValueError):
        GrowthController(m, torch.optim.SGD(m.parameters(), lr=0.1), schedule=[(0, "bogus", {})]).maybe_grow(0, 1.0)
