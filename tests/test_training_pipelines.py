"""ACT-V verifier, reward functions, GRPO and the phase-2/3/ACT-V trainers on CPU."""

import copy
import math
import random

import pytest
import torch

from genesis.model import HLRT, HLRTConfig
from genesis.training.grpo import GRPOConfig, GRPOTrainer
from genesis.training.reward_functions import (CompositeReward, CorrectnessReward, FormatReward,
                                               InformationGainReward, completion_logprobs)
from genesis.training.train_actv import ACTVConfig, ACTVTrainer
from genesis.training.train_phase2_rl import RLPretrainer
from genesis.training.train_phase3_flywheel import FlywheelTrainer
from genesis.verifier import (NegativeGenerator, ReplayBuffer, VerificationDistillation, VerificationHead,
                              VerifierModel)
from olympus.data.flywheel_buffer import FlywheelBuffer
from olympus.data.tokenizer import TokenizerWrapper

TINY = dict(
    vocab_size=300, d_model=64, tier1_num_layers=2, tier1_num_heads=4, tier1_d_ff=128,
    gate1_chunk_size=4, num_latent_vectors=2, latent_pool_num_heads=2,
    tier2_d_model=64, tier2_num_layers=1, tier2_num_heads=4, tier2_d_ff=128,
    tier3_d_model=64, tier3_num_layers=1, tier3_num_heads=4, tier3_d_ff=128, tier3_recurrence_steps=2,
)


def _hlrt(seed=0):
    torch.manual_seed(seed)
    return HLRT(HLRTConfig(**TINY))


def _tok():
    return TokenizerWrapper(backend="char", vocab_size=300)


# ------------------------------------------------------------------ verifier
def test_verifier_model_masked_pooling_ignores_padding():
    torch.manual_seed(0)
    v = VerifierModel(vocab_size=300, d_model=32, num_layers=2, num_heads=4, d_ff=64, max_seq_len=64).eval()
    ids = torch.randint(0, 300, (1, 12))
    mask = torch.ones(1, 12)
    mask[:, 8:] = 0
    a = v(ids, mask)["pooled_output"]
    ids2 = ids.clone()
    ids2[:, 8:] = 7  # different padding content, same mask
    b = v(ids2, mask)["pooled_output"]
    torch.testing.assert_close(a, b)
    assert v(ids)["hidden_states"].shape == (1, 12, 32)


def test_verification_head_loss_matches_per_head_bce():
    torch.manual_seed(0)
    h = VerificationHead(16)
    x = torch.randn(5, 16)
    s = h(x)
    for i, k in enumerate(("factual_score", "logical_score", "stylistic_score", "overall_score")):
        head = getattr(h, k.replace("_score", "_head"))
        torch.testing.assert_close(s[k], head(x))
    lab = {"factual_score": torch.ones(5, 1), "logical_score": torch.zeros(5, 1)}
    want = (torch.nn.functional.binary_cross_entropy(s["factual_score"], lab["factual_score"])
            + torch.nn.functional.binary_cross_entropy(s["logical_score"], lab["logical_score"])
            + torch.nn.functional.binary_cross_entropy(s["overall_score"], torch.full((5, 1), 0.4)))
    torch.testing.assert_close(h.compute_loss(s, lab), want)


@pytest.mark.parametrize("kind", ["entity_swap", "negation_insertion", "number_perturbation",
                                  "fact_substitution", "temporal_shift"])
def test_negative_generator_labels_mark_changes(kind):
    random.seed(3)
    ng = NegativeGenerator(vocab_size=20000)
    ids = torch.randint(0, 20000, (60,))
    ids[5] = 8091  # a temporal marker
    out, labels, locs = ng.corrupt(ids, kind)
    assert out.shape == labels.shape and len(locs) > 0
    assert bool((labels == 0).any())
    if out.numel() == ids.numel() and kind != "fact_substitution":
        changed = (out != ids)
        assert bool((labels[changed] == 0).all())
        assert bool(changed[labels == 0].all())
    if kind == "temporal_shift":
        assert int(out[5]) == 10643


def test_negative_generator_batch_and_replay_buffer():
    random.seed(0)
    ng = NegativeGenerator(vocab_size=1000)
    ids, labels = ng.batch_corrupt(torch.randint(0, 1000, (4, 30)))
    assert ids.shape == labels.shape and ids.shape[0] == 4 and ids.shape[1] >= 30
    rb = ReplayBuffer(3)
    for i in range(5):
        rb.add(torch.full((4,), i), {"overall_score": torch.tensor([0.5])})
    assert rb.size == 3 and sorted(int(e["input_ids"][0]) for e in rb.sample(10)) == [2, 3, 4]
    rb.add_batch(torch.zeros(2, 4, dtype=torch.long), {"overall_score": torch.ones(2, 1)})
    assert rb.size == 3
    with pytest.raises(ValueError):
        ReplayBuffer(0)


def test_distillation_losses():
    torch.manual_seed(0)
    d = VerificationDistillation(8, 4, shared_dim=6)
    g, v = torch.randn(3, 8, requires_grad=True), torch.randn(3, 4)
    loss = d(g, v)
    loss.backward()
    assert g.grad is not None and d.proj_V.weight.grad is None
    gl, vl = torch.randn(2, 5), torch.randn(2, 5)
    T = 2.0
    ref = (torch.softmax(vl / T, -1) * (torch.log_softmax(vl / T, -1) - torch.log_softmax(gl / T, -1))).sum(-1).mean() * T * T
    torch.testing.assert_close(d.temperature_scaled_loss(gl, vl, T), ref)


# ------------------------------------------------------------------- rewards
def test_correctness_and_format_rewards():
    c = CorrectnessReward({"q": "42", "r": "Paris"})
    assert c("q", "so the answer is 42.") == 1.0
    assert c("q", "answer: 42.0") == 1.0
    assert c("q", "I think 42") == 0.5
    assert c("q", "answer is 41") == 0.0
    assert c("r", "answer: paris") == 1.0
    assert c("unknown", "answer: 1") == 0.0
    f = FormatReward(required_sections=[r"step \d"])
    assert f("", "<|reason_start|>step 1<|reason_end|>") == pytest.approx(0.75)
    assert f("", "<|reason_start|><|reason_end|>") == pytest.approx(0.125)
    assert f("", "<|reason_start|> only") == pytest.approx(0.05)
    assert f("", "   ") == 0.0
    comp = CompositeReward([(c, 1.0), (f, 3.0)])
    assert comp("q", "answer is 42") == pytest.approx((1.0 + 0.0) / 4.0)
    assert CompositeReward([(c, 1.0), (f, 3.0)], normalize=False)("q", "answer is 42") == pytest.approx(1.0)


def test_completion_logprobs_matches_unpadded_forward():
    m = _hlrt().eval()
    pre, comp = [[1, 2, 3], [4, 5]], [[6, 7], [8, 9, 10, 11]]
    s, n = completion_logprobs(m, pre, comp, torch.device("cpu"))
    for i in range(2):
        ids = torch.tensor([pre[i] + comp[i]])
        lp = torch.log_softmax(m(ids)["logits"][0, :-1].float(), -1).gather(-1, ids[0, 1:, None]).squeeze(-1)
        want = lp[len(pre[i]) - 1:].sum()
        torch.testing.assert_close(s[i], want, atol=1e-4, rtol=1e-4)
        assert int(n[i]) == len(comp[i])


def test_information_gain_reward_is_bounded():
    tok = _tok()
    r = InformationGainReward(_hlrt(), tok)
    vals = r.score_batch(["hello ", "abc"], ["world", ""])
    assert -1.0 <= vals[0] <= 1.0 and vals[1] == -1.0
    assert r("hello ", "world") == pytest.approx(vals[0], abs=1e-5)


# ---------------------------------------------------------------------- GRPO
def test_grpo_advantages_and_loss():
    t = GRPOTrainer(_hlrt(), _hlrt(), lambda p, c: 0.0, GRPOConfig(group_size=4))
    r = torch.tensor([[1.0, 2.0, 3.0, 4.0], [5.0, 5.0, 5.0, 5.0]])
    a = t.compute_advantages(r)
    torch.testing.assert_close(a[0], (r[0] - 2.5) / r[0].std())
    assert torch.all(a[1] == 0)
    lp = torch.tensor([[0.1, -0.3]])
    ref = torch.tensor([[0.0, 0.0]])
    adv = torch.tensor([[1.0, -1.0]])
    loss, m = t.compute_loss(lp, ref, adv)
    ratio = lp.exp()
    pol = -torch.min(ratio * adv, ratio.clamp(0.8, 1.2) * adv).mean()
    kl = ((ratio - 1) - lp).mean()
    torch.testing.assert_close(loss, pol + 0.1 * kl)
    assert m["clip_fraction"] == pytest.approx(0.5)


def test_grpo_step_updates_policy_only():
    torch.manual_seed(0)
    pol = _hlrt(0)
    ref = copy.deepcopy(pol)
    tok = _tok()
    opt = torch.optim.SGD(pol.parameters(), lr=1e-2)
    t = GRPOTrainer(pol, ref, FormatReward(), GRPOConfig(group_size=3, max_completion_tokens=5))
    before = [p.detach().clone() for p in ref.parameters()]
    m = t.step({"prompts": ["ab", "xyz"], "tokenizer": tok, "optimizer": opt})
    assert math.isfinite(m["loss"]) and set(m) >= {"reward_mean", "kl_div", "clip_fraction", "mean_ratio"}
    assert all(torch.equal(a, b) for a, b in zip(before, ref.parameters()))
    groups = t.generate_group(["ab"], tok)
    assert len(groups) == 1 and len(groups[0]) == 3


# ------------------------------------------------------------------ trainers
def test_rl_pretrainer_mixes_objectives():
    torch.manual_seed(0)
    pol = _hlrt(0)
    opt = torch.optim.AdamW(pol.parameters(), lr=1e-3)
    tr = RLPretrainer(pol, copy.deepcopy(pol), FormatReward(), opt,
                      {"device": "cpu", "gradient_accumulation_steps": 1, "grpo_group_size": 2,
                       "grpo_max_tokens": 4, "rl_mix": 0.25})
    w0 = pol.embeddings.embedding.weight.detach().clone()
    m = tr.train_step({"input_ids": torch.randint(0, 300, (2, 16)), "prompts": ["hi"], "tokenizer": _tok()})
    assert math.isfinite(m["ntp_loss"]) and m["total_loss"] == pytest.approx(0.75 * m["ntp_loss"] + 0.25 * m["rl_loss"])
    assert tr.orchestrator.global_step == 1
    assert not torch.equal(w0, pol.embeddings.embedding.weight)


def test_flywheel_step_stores_and_mixes():
    torch.manual_seed(0)
    m = _hlrt(0)
    buf = FlywheelBuffer(max_size=16, reward_threshold=-1e9)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    tr = FlywheelTrainer(m, buf, lambda model, c, t: torch.ones(c.size(0)), opt,
                         {"device": "cpu", "gradient_accumulation_steps": 1, "max_trace_tokens": 4,
                          "tokenizer": _tok(), "trace_mix_ratio": 0.5})
    out = tr.flywheel_step({"input_ids": torch.randint(0, 300, (4, 16))})
    assert out["traces_generated"] == 4 and out["traces_stored"] == 4 and out["buffer_size"] == 4
    assert out["avg_reward"] == pytest.approx(1.0)
    mixed = tr._mix_with_buffer({"input_ids": torch.randint(0, 300, (4, 16))})["input_ids"]
    assert mixed.shape == (4, 16)
    e = buf.sample(1)[0]
    assert len(e["metadata"]["token_ids"]) == 8 + 4


def test_actv_co_training_and_distillation():
    random.seed(0)
    torch.manual_seed(0)
    gen = _hlrt(0)
    ver = VerifierModel(vocab_size=300, d_model=32, num_layers=1, num_heads=4, d_ff=64, max_seq_len=64)
    tr = ACTVTrainer(gen, ver, NegativeGenerator(vocab_size=300, negation_tokens=[1, 2, 3], temporal_map={4: 5, 5: 4}),
                     ReplayBuffer(64),
                     ACTVConfig(distill_interval=2, replay_min_size=2, distillation_shared_dim=8))
    ids = torch.randint(0, 300, (2, 16))
    m1 = tr.co_training_step({"input_ids": ids, "labels": ids})
    assert tr.replay_buffer.size == 2 and "distillation_loss" not in m1
    m2 = tr.co_training_step({"input_ids": ids, "labels": ids})
    assert m2["v_replay_loss"] > 0 and "distillation_loss" in m2
    assert m2["g_ntp_loss"] > 0 and 0 <= m2["g_v_scores"]["overall_score"] <= 1


def test_init_distributed_sets_async_error_handling_and_timeout(monkeypatch):
    """Two gloo ranks come up through the trainer's initialiser with the
    watchdog's error handling switched on and the timeout from the environment."""
    from tests.dist_utils import run_ranks

    monkeypatch.delenv("TORCH_NCCL_ASYNC_ERROR_HANDLING", raising=False)
    monkeypatch.setenv("LRB_PG_TIMEOUT_S", "45")
    for res in run_ranks(_init_case, 2):
        assert res == ("1", 45.0)


def _init_case(rank, world):
    import os

    import torch.distributed as dist

    from genesis.training.train_phase1_distributed import init_distributed

    dist.destroy_process_group()  # the harness initialised one; the trainer's initialiser makes its own
    os.environ.pop("TORCH_NCCL_ASYNC_ERROR_HANDLING", None)
    init_distributed()
    import torch
    from torch.distributed.distributed_c10d import _get_default_group

    backend = _get_default_group()._get_backend(torch.device("cpu"))
    return os.environ["TORCH_NCCL_ASYNC_ERROR_HANDLING"], backend.options._timeout.total_seconds()
