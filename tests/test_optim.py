"""Muon, MuonAdamWHybrid and WSDScheduler (CPU)."""

import math

import pytest
import torch
import torch.nn as nn

from olympus.optim import Muon, MuonAdamWHybrid, WSDScheduler


def _reference_ns(G, steps=5, eps=1e-7):
    """The reference iteration verbatim in math: tall orientation, X X^T Gram."""
    transposed = G.shape[0] < G.shape[1]
    if transposed:
        G = G.T
    X = G / (G.norm() + eps)
    a, b, c = 3.4445, -4.7750, 2.0315
    for _ in range(steps):
        A = X @ X.T
        X = a * X + b * (A @ X) + c * (A @ (A @ X))
    return X.T if transposed else X


@pytest.mark.parametrize("shape", [(64, 64), (32, 96), (96, 32)])
def test_newton_schulz_short_side_gram_equals_reference(shape):
    torch.manual_seed(0)
    G = torch.randn(*shape, dtype=torch.float64)
    got = Muon._newton_schulz(G.float(), steps=5).double()
    ref = _reference_ns(G, steps=5)
    assert (got - ref).abs().max().item() < 1e-4


def test_newton_schulz_orthogonality():
    torch.manual_seed(0)
    Q = Muon._newton_schulz(torch.randn(64, 64), steps=5)
    assert (Q @ Q.T - torch.eye(64)).abs().max().item() < 0.5
    assert Muon._newton_schulz(torch.randn(32, 64)).shape == (32, 64)


def test_muon_rejects_non_2d():
    with pytest.raises(ValueError):
        Muon([nn.Parameter(torch.randn(4))])
    with pytest.raises(ValueError):
        Muon([nn.Parameter(torch.randn(4, 4))], lr=-1)


def _reference_muon_update(p, g, buf, lr, mu, wd):
    if wd:
        p = p * (1 - lr * wd)
    buf = buf * mu + g
    u = g + mu * buf
    o = _reference_ns(u.double()).float()
    o = o * (g.norm() / (o.norm() + 1e-8))
    return p - lr * o, buf


def test_muon_step_matches_reference_update():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(48, 32))
    opt = Muon([p], lr=0.02, momentum=0.95, weight_decay=0.1)
    ref_p, ref_buf = p.detach().clone(), torch.zeros(48, 32)
    for _ in range(3):
        g = torch.randn(48, 32)
        p.grad = g.clone()
        opt.step()
        ref_p, ref_buf = _reference_muon_update(ref_p, g, ref_buf, 0.02, 0.95, 0.1)
    torch.testing.assert_close(p.detach(), ref_p, atol=1e-5, rtol=1e-4)
    torch.testing.assert_close(opt.state[p]["momentum_buffer"], ref_buf)


def test_hybrid_routing_and_state_layout():
    torch.manual_seed(0)
    emb = nn.Parameter(torch.randn(1000, 16))   # aspect 62 -> AdamW
    w = nn.Parameter(torch.randn(32, 16))        # Muon
    b = nn.Parameter(torch.randn(16))            # AdamW
    opt = MuonAdamWHybrid([emb, w, b])
    for p in (emb, w, b):
        p.grad = torch.randn_like(p)
    opt.step()
    assert opt.state[w]["type"] == "muon" and set(opt.state[w]) == {"type", "momentum_buffer"}
    for p in (emb, b):
        assert opt.state[p]["type"] == "adamw" and opt.state[p]["step"] == 1
        assert set(opt.state[p]) == {"type", "step", "exp_avg", "exp_avg_sq"}
    keys = set(opt.state_dict()["param_groups"][0])
    assert {"lr_muon", "lr_adamw", "momentum", "betas", "eps", "weight_decay_muon", "weight_decay_adamw",
            "ns_steps", "muon_max_aspect_ratio", "params"} <= keys


def test_hybrid_adamw_matches_torch_math():
    torch.manual_seed(0)
    p = nn.Parameter(torch.randn(20))
    ref = p.detach().clone()
    opt = MuonAdamWHybrid([p], lr_adamw=1e-2, weight_decay_adamw=0.1)
    m = torch.zeros(20)
    v = torch.zeros(20)
    for t in range(1, 4):
        g = torch.randn(20)
        p.grad = g.clone()
        opt.step()
        ref = ref * (1 - 1e-2 * 0.1)
        m = 0.9 * m + 0.1 * g
        v = 0.999 * v + 0.001 * g * g
        ref = ref - 1e-2 * (m / (1 - 0.9 ** t)) / ((v / (1 - 0.999 ** t)).sqrt() + 1e-8)
    torch.testing.assert_close(p.detach(), ref, atol=1e-6, rtol=1e-6)


def test_wsd_schedule_shape_and_state():
    opt = torch.optim.SGD([nn.Parameter(torch.zeros(1))], lr=1.0)
    s = WSDScheduler(opt, base_lr=1.0, min_lr=0.1, warmup_steps=10, total_steps=100, decay_start=80,
                     post_growth_warmup_steps=5)
    assert s.get_lr(0) == 0.0 and abs(s.get_lr(5) - 0.5) < 1e-9 and s.get_lr(50) == 1.0
    assert abs(s.get_lr(100) - 0.1) < 1e-9 and 0.1 < s.get_lr(90) < 1.0
    s.notify_growth(50)
    assert s.get_lr(50) == 0.0 and abs(s.get_lr(52) - 0.4) < 1e-9 and s.get_lr(60) == 1.0
    for _ in range(12):
        s.step()
    assert opt.param_groups[0]["lr"] == s.last_lr
    sd = s.state_dict()
    assert set(sd) == {"step_count", "growth_step", "last_lr", "base_lr", "min_lr", "warmup_steps", "total_steps",
                       "decay_start", "post_growth_warmup_steps"}
    s2 = WSDScheduler(opt)
    s2.load_state_dict(sd)
    assert s2.get_lr() == s.get_lr()


def test_wsd_hybrid_lrs_reference_behaviour_and_flag():
    w = nn.Parameter(torch.randn(8, 8))
    opt = MuonAdamWHybrid([w], lr_muon=0.02, lr_adamw=3e-4)
    s = WSDScheduler(opt, base_lr=1.0, warmup_steps=10, total_steps=100)
    s.step(); s.step(); s.step()
    assert opt.param_groups[0]["lr_muon"] == 0.02  # reference: schedule never reaches the hybrid
    opt2 = MuonAdamWHybrid([w], lr_muon=0.02, lr_adamw=3e-4)
    s2 = WSDScheduler(opt2, base_lr=1.0, warmup_steps=10, total_steps=100, drive_hybrid_lrs=True)
    s2.step(); s2.step(); s2.step()
    assert math.isclose(opt2.param_groups[0]["lr_muon"], 0.02 * 0.2)
    assert math.isclose(opt2.param_groups[0]["lr_adamw"], 3e-4 * 0.2)
