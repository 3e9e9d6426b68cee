"""The shipped YAML configurations (nested model schema) build exactly the
named presets."""

import os

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("name,preset", [("genesis_1b", "genesis-1b"), ("genesis_7b_nvfp4", "genesis-7b-nvfp4"),
                                         ("genesis_40b_moe", "genesis-40b-moe")])
def test_yaml_matches_preset(name, preset):
    from llm_research_b200.models.presets import build_hlrt_config
    from olympus.utils.config import hlrt_config_from_yaml

    got = hlrt_config_from_yaml(os.path.join(ROOT, "genesis", "training", "configs", f"{name}.yaml"))
    want = build_hlrt_config(preset)
    assert got.to_dict() == want.to_dict()


_TRAIN_YAML = """
model:
  vocab_size: 256
  max_seq_len: 64
  tier1: {layers: 2, d_model: 64, heads: 4, d_ff: 128}
  tier2: {layers: 0, d_model: 64, heads: 4, latent_vectors_per_chunk: 8, chunk_size: 32, max_seq_len: 64,
          latent_pool_heads: 4}
  tier3: {layers: 0, d_model: 64, heads: 4, recurrence_steps: 1, max_seq_len: 64}
optimizer: {muon_lr: 0.01, adamw_lr: 1.0e-3, muon_momentum: 0.9, adamw_betas: [0.9, 0.95], weight_decay: 0.1,
            ns_iterations: 3}
scheduler: {warmup_steps: 1, stable_steps: 2, decay_steps: 1, min_lr: 1.0e-5}
training: {batch_size: 2, gradient_accumulation_steps: 1, max_steps: 3, gradient_clip: 0.5,
           checkpoint_interval: 100, log_interval: 1, seq_len: 64}
hardware: {device: cpu, precision: fp32}
"""


def test_trainer_settings_and_dotted_overrides(tmp_path):
    from olympus.utils.config import hlrt_config_from_yaml, load_config, parse_overrides, trainer_settings_from_yaml

    path = tmp_path / "run.yaml"
    path.write_text(_TRAIN_YAML)
    ov = parse_overrides(["model.tier1.layers=1", "optimizer.adamw_betas=[0.8, 0.9]", "training.max_steps=2"])
    assert ov == {"model.tier1.layers": 1, "optimizer.adamw_betas": [0.8, 0.9], "training.max_steps": 2}
    cfg = load_config(str(path), ov)
    assert hlrt_config_from_yaml(cfg).tier1_num_layers == 1
    s = trainer_settings_from_yaml(cfg)
    assert s["optimizer_kwargs"] == {"lr_muon": 0.01, "lr_adamw": 1e-3, "momentum": 0.9, "betas": (0.8, 0.9),
                                     "weight_decay_adamw": 0.1, "ns_steps": 3}
    assert s["scheduler_kwargs"] == {"base_lr": 1e-3, "min_lr": 1e-5, "warmup_steps": 1, "decay_steps": 1,
                                     "decay_start": 3, "total_steps": 4}
    assert s["trainer"]["max_steps"] == 2 and s["trainer"]["max_grad_norm"] == 0.5
    with pytest.raises(ValueError):
        parse_overrides(["no_equals_sign"])


def test_distributed_trainer_cli_runs_from_yaml(tmp_path):
    from genesis.training.train_phase1_distributed import main

    path = tmp_path / "run.yaml"
    path.write_text(_TRAIN_YAML)
    ck = tmp_path / "ck"
    main(["--config", str(path), "--set", "model.tier1.layers=1", "--max-steps", "2", "--checkpoint-dir", str(ck)])
    state = torch.load(ck / "checkpoint_final.pt", weights_only=False)
    assert state["global_step"] == 2
    n_blocks = {k.split(".")[2] for k in state["models"]["hlrt"] if k.startswith("tier1.layers.")}
    assert n_blocks == {"0"}


def test_resumable_sampler_continues_mid_epoch():
    from olympus.data.resumable_sampler import ResumableDistributedSampler

    full = [list(ResumableDistributedSampler(50, 2, r, seed=3)) for r in range(2)]
    assert sorted(full[0] + full[1]) == sorted(set(full[0] + full[1])) and len(full[0]) == 25
    s = ResumableDistributedSampler(50, 2, 1, seed=3)
    s.advance(6)
    t = ResumableDistributedSampler(50, 2, 1, seed=3)
    t.load_state_dict(s.state_dict())
    assert list(t) == full[1][6:] and len(t) == 19
    t.set_epoch(1)
    assert len(t) == 25 and list(t) != full[1]


def test_trainer_resume_sees_the_remaining_samples(tmp_path):
    """Stop after 3 steps of an epoch, resume from the checkpoint: the resumed
    trainer's loader yields exactly the batches an uninterrupted run had left."""
    from genesis.model.hlrt import HLRT
    from genesis.training.train_phase1_distributed import DistributedBootstrapTrainer
    from llm_research_b200.models.presets import build_hlrt_config
    from olympus.data.packed_dataset import SyntheticTokenDataset

    cfg = build_hlrt_config("toy")
    ds = SyntheticTokenDataset(16, 32, cfg.vocab_size)

    def trainer():
        torch.manual_seed(0)
        return DistributedBootstrapTrainer(HLRT(cfg), config={"log_interval": 100, "save_interval": 0,
                                                              "gradient_accumulation_steps": 1,
                                                              "max_steps": 3, "checkpoint_dir": str(tmp_path)})

    a = trainer()
    loader = a.make_dataloader(ds, batch_size=2, num_workers=0)
    expect = [b["input_ids"].clone() for b in loader]
    a.train_epoch(loader)  # stops after 3 steps
    a.save_checkpoint(str(tmp_path / "c.pt"))
    b = trainer()
    b.load_checkpoint(str(tmp_path / "c.pt"))
    rest = [x["input_ids"] for x in b.make_dataloader(ds, batch_size=2, num_workers=0)]
    assert len(rest) == len(expect) - 3
    for x, y in zip(rest, expect[3:]):
        assert torch.equal(x, y)


def _resume_case(rank, world, d):
    from genesis.model.hlrt import HLRT
    from genesis.training.train_phase1_distributed import DistributedBootstrapTrainer
    from llm_research_b200.models.presets import build_hlrt_config
    from olympus.data.packed_dataset import SyntheticTokenDataset

    cfg = build_hlrt_config("toy")
    ds = SyntheticTokenDataset(16, 32, cfg.vocab_size)

    def trainer():
        torch.manual_seed(0)
        return DistributedBootstrapTrainer(HLRT(cfg), config={"log_interval": 100, "save_interval": 0, "max_steps": 2,
                                                              "gradient_accumulation_steps": 1, "checkpoint_dir": d})

    a = trainer()
    loader = a.make_dataloader(ds, batch_size=2, num_workers=0)
    expect = [b["input_ids"].clone() for b in loader]
    a.train_epoch(loader)
    a.save_checkpoint(os.path.join(d, "c.pt"))
    b = trainer()
    b.load_checkpoint(os.path.join(d, "c.pt"))
    rest = [x["input_ids"] for x in b.make_dataloader(ds, batch_size=2, num_workers=0)]
    return expect, rest


def test_trainer_resume_mid_epoch_two_ranks(tmp_path):
    from tests.dist_utils import run_ranks

    res = run_ranks(_resume_case, 2, str(tmp_path))
    for expect, rest in res:
        assert len(expect) == 4 and len(rest) == 2
        assert all(torch.equal(x, y) for x, y in zip(rest, expect[2:]))
    assert not torch.equal(res[0][0][0], res[1][0][0])  # the ranks read different samples
