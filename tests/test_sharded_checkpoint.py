"""Sharded asynchronous checkpoints: save on 2 gloo ranks, consolidate to full
tensors, reload into the same layout and into a different world size."""

import torch

from tests.dist_utils import run_ranks


def _model():
    from genesis.model import HLRT, HLRTConfig

    torch.manual_seed(0)
    return HLRT(HLRTConfig(vocab_size=128, d_model=32, tier1_num_layers=2, tier1_num_heads=2, tier1_d_ff=64,
                           gate1_chunk_size=4, num_latent_vectors=2, latent_pool_num_heads=2, tier2_d_model=32,
                           tier2_num_layers=1, tier2_num_heads=2, tier2_d_ff=64, tier3_d_model=32,
                           tier3_num_layers=1, tier3_num_heads=2, tier3_d_ff=64))


def _save(rank, world, d):
    from llm_research_b200.parallel import checkpoint as ck
    from llm_research_b200.parallel.fsdp import FlatShardEngine
    from olympus.optim import MuonAdamWHybrid

    eng = FlatShardEngine(_model())
    defaults = MuonAdamWHybrid([torch.nn.Parameter(torch.zeros(2, 2))], lr_muon=0.02, lr_adamw=1e-3).defaults
    opt = eng.make_optimizer(MuonAdamWHybrid, defaults)
    ids = torch.randint(0, 128, (2, 16), generator=torch.Generator().manual_seed(rank))
    out = eng(ids)
    torch.nn.functional.cross_entropy(out["logits"].reshape(-1, 128), ids.reshape(-1)).backward()
    opt.step()
    opt.zero_grad()
    ck.save_sharded(eng, opt, d, header={"global_step": 1, "phase": "bootstrap"})
    ck.wait()
    return eng.full_state_dict()


def _load(rank, world, d):
    from llm_research_b200.parallel import checkpoint as ck
    from llm_research_b200.parallel.fsdp import FlatShardEngine
    from olympus.optim import MuonAdamWHybrid

    eng = FlatShardEngine(_model())
    defaults = MuonAdamWHybrid([torch.nn.Parameter(torch.zeros(2, 2))], lr_muon=0.02, lr_adamw=1e-3).defaults
    opt = eng.make_optimizer(MuonAdamWHybrid, defaults)
    header = ck.load_sharded(eng, opt, d)
    return header, eng.full_state_dict()


def test_sharded_save_consolidate_reload(tmp_path):
    from llm_research_b200.parallel.checkpoint import consolidate

    d = str(tmp_path / "ck")
    saved = run_ranks(_save, 2, d)[0]
    full = consolidate(d)
    assert full["world_size"] == 2 and full["global_step"] == 1
    for k, v in saved.items():
        torch.testing.assert_close(full["models"]["model"][k], v)
    assert any("momentum_buffer" in k or "momentum" in st for st in full["optimizer_state"]["model"].values() for k in st)
    header, again = run_ranks(_load, 2, d)[0]
    assert header["phase"] == "bootstrap"
    for k, v in saved.items():
        torch.testing.assert_close(again[k], v)
    _, single = run_ranks(_load, 1, d)[0]  # different world size: consolidated on load
    for k, v in saved.items():
        torch.testing.assert_close(single[k], v)


def _orch_resume(rank, world, d):
    from tests.test_engine import _data, _toy_model, _train

    data = _data()
    per = data.shape[0] // world
    batch = [data[rank * per:(rank + 1) * per]]
    _, orch = _train(_toy_model(), batch, engine=True, steps=2)
    orch.save_sharded_checkpoint(d)  # asynchronous: training continues
    orch.step({"input_ids": batch[0]})
    cont = orch._models["hlrt"].model.full_state_dict()
    _, orch2 = _train(_toy_model(), batch, engine=True, steps=0)
    head = orch2.load_sharded_checkpoint(d)
    orch2.step({"input_ids": batch[0]})
    resumed = orch2._models["hlrt"].model.full_state_dict()
    return head["global_step"], cont, resumed


def test_orchestrator_sharded_resume_and_consolidation(tmp_path):
    from llm_research_b200.parallel.checkpoint import consolidate_checkpoint, main

    d = str(tmp_path / "orch")
    step, cont, resumed = run_ranks(_orch_resume, 2, d)[0]
    assert step == 2
    for k, v in cont.items():  # momentum / Adam state restored: the resumed step equals the continued one
        torch.testing.assert_close(resumed[k], v, atol=1e-6, rtol=1e-5, msg=k)
    full = consolidate_checkpoint(d)
    assert full["global_step"] == 2 and full["world_size"] == 2
    assert set(cont) <= set(full["models"]["hlrt"])
    out = str(tmp_path / "full.pt")
    main([d, out])
    assert torch.load(out, weights_only=False)["phase"] == full["phase"]


def test_checkpoint_restores_rng_streams(tmp_path):
    """A resumed run draws the same random numbers as an uninterrupted one
    (Python, NumPy and torch generators are saved with the checkpoint)."""
    import random

    import numpy as np
    import torch.nn as nn

    from olympus.core.training_orchestrator import ModelConfig, TrainingOrchestrator

    torch.manual_seed(0)
    model = nn.Linear(4, 4)
    orch = TrainingOrchestrator(device="cpu")
    orch.add_model(ModelConfig(name="m", model=model, optimizer=torch.optim.SGD(model.parameters(), lr=0.1)))
    random.seed(1), np.random.seed(2), torch.manual_seed(3)
    path = str(tmp_path / "c.pt")
    orch.save_checkpoint(path)
    expect = (random.random(), float(np.random.rand()), torch.rand(3))
    random.seed(9), np.random.seed(9), torch.manual_seed(9)
    orch.load_checkpoint(path)
    got = (random.random(), float(np.random.rand()), torch.rand(3))
    assert got[0] == expect[0] and got[1] == expect[1] and torch.equal(got[2], expect[2])
    torch.load(path, weights_only=True)  # plain tensors, numbers and strings only
