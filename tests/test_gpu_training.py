"""End-to-end training on the GPU through the public trainer API."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _trainer(cfg, device, precision, seed=0, accum=2):
    from genesis.model.hlrt import HLRT
    from genesis.training.train_phase1_bootstrap import BootstrapTrainer
    from olympus.data.tokenizer import TokenizerWrapper
    from olympus.optim import MuonAdamWHybrid, WSDScheduler

    torch.manual_seed(seed)
    model = HLRT(cfg)
    opt = MuonAdamWHybrid(model.parameters(), lr_muon=0.02, lr_adamw=3e-3)
    sched = WSDScheduler(opt, base_lr=3e-3, warmup_steps=0, total_steps=100)
    return BootstrapTrainer(model, opt, sched, TokenizerWrapper("char", vocab_size=cfg.vocab_size),
                            {"device": device, "gradient_accumulation_steps": accum, "precision": precision})


def test_gpu_bf16_engine_tracks_cpu_fp32_oracle():
    from llm_research_b200.models.presets import build_hlrt_config

    cfg = build_hlrt_config("toy")
    ids = torch.randint(0, cfg.vocab_size, (2, 128), generator=torch.Generator().manual_seed(1))
    cpu = _trainer(cfg, "cpu", "fp32")
    gpu = _trainer(cfg, "cuda", "bf16")
    lc, lg = [], []
    for _ in range(6):
        lc.append(float(cpu.train_step({"input_ids": ids})["loss"]))
        lg.append(float(gpu.train_step({"input_ids": ids})["loss"]))
    assert abs(lc[0] - lg[0]) < 0.05, (lc, lg)
    assert lg[-1] < lg[0]
    assert max(abs(a - b) for a, b in zip(lc, lg)) < 0.1, (lc, lg)


def test_gpu_genesis_1b_layer_shapes_step():
    """One optimizer step of a 2-layer slice of the 1B geometry (d 2048, seq 4096)."""
    from llm_research_b200.models.presets import build_hlrt_config

    cfg = build_hlrt_config("genesis-1b")
    cfg.tier1_num_layers = 2
    tr = _trainer(cfg, "cuda", "bf16", accum=1)
    ids = torch.randint(0, cfg.vocab_size, (1, 4096), device="cuda")
    l0 = float(tr.train_step({"input_ids": ids})["loss"])
    l1 = float(tr.train_step({"input_ids": ids})["loss"])
    assert l0 == l0 and l1 < l0
