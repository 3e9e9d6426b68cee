"""The CPU plumbing configuration: tiny GENESIS dense HLRT (4 layers per tier,
d_model 256, 4 heads, SwiGLU 1024, vocab 32000, a PHMA read of 1024 slots x 256
with top-8), fp32, 2 gloo ranks, batch 4 x seq 256 of uniform token ids from
seed 0, N(0, 0.02) init, Muon on 2-D weights and AdamW elsewhere, 10 steps."""

import torch

from tests.dist_utils import run_ranks


def _rank(rank, world):
    from genesis.model.hlrt import HLRT
    from genesis.training.train_phase1_bootstrap import ntp_objective
    from llm_research_b200.models.presets import build_hlrt_config
    from olympus.core.training_orchestrator import ModelConfig, ObjectiveConfig
    from olympus.distributed.distributed_orchestrator import DistributedTrainingOrchestrator
    from olympus.distributed.fsdp_wrapper import FSDPConfig
    from olympus.optim import MuonAdamWHybrid

    cfg = build_hlrt_config("tiny")
    assert cfg.tier1_memory_every and cfg.memory_slots == 1024 and cfg.memory_top_k == 8
    torch.manual_seed(0)
    model = HLRT(cfg)
    opt = MuonAdamWHybrid(model.parameters(), lr_muon=0.02, lr_adamw=1e-3)
    orch = DistributedTrainingOrchestrator(
        fsdp_config=FSDPConfig(mixed_precision="fp32", activation_checkpointing=False), device=torch.device("cpu"),
        world_size=world)
    orch.add_model(ModelConfig("hlrt", model, opt, max_grad_norm=1.0))
    orch.add_objective(ObjectiveConfig("ntp", ntp_objective))
    ids = torch.randint(0, cfg.vocab_size, (4, 256), generator=torch.Generator().manual_seed(0))
    mine = ids[rank * 2:(rank + 1) * 2]
    losses = [float(orch.step({"input_ids": mine})["total"]) for _ in range(10)]
    sd = orch._models["hlrt"].model.full_state_dict()
    return losses, {k: v.clone() for k, v in list(sd.items())[:8]}


def test_tiny_config_two_gloo_ranks_ten_steps():
    res = run_ranks(_rank, 2)
    for losses, _ in res:
        assert all(l == l and l < 20 for l in losses)
        assert losses[-1] < losses[0]
    for k, v in res[0][1].items():  # both ranks hold the same weights after 10 steps
        torch.testing.assert_close(res[1][1][k], v)
