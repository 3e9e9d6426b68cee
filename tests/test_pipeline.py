"""Pipeline parallelism over the Tier-1 trunk: 2 gloo stages, 1F1B over 4
micro-batches, against one process running the same micro-batches."""

import torch
import torch.nn.functional as F

from tests.dist_utils import run_ranks


def _model():
    from genesis.model.hlrt import HLRT
    from llm_research_b200.models.presets import build_hlrt_config

    cfg = build_hlrt_config("toy")
    cfg.tier1_num_layers = 4
    torch.manual_seed(0)
    return HLRT(cfg), cfg


def _loss(out, ids):
    logits = out["logits"]
    return F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), ids[:, 1:].reshape(-1)) \
        + out["aux_loss"]


def _batches(cfg):
    g = torch.Generator().manual_seed(3)
    return [torch.randint(0, cfg.vocab_size, (1, 32), generator=g) for _ in range(4)]


def _stage(rank, world):
    from llm_research_b200.parallel.pipeline import PipelineStage

    m, cfg = _model()
    st = PipelineStage(m)
    mb = _batches(cfg)
    loss = st.train_step(mb, _loss, act_shape=(1, 32, cfg.d_model), act_dtype=torch.float32)
    st.sync_tied_gradients()
    grads = {n: p.grad.clone() for n, p in m.named_parameters() if n in st.owned_names and p.grad is not None}
    return (float(loss) if loss is not None else None), grads, st.layer_range


def test_pipeline_two_stages_matches_single_process():
    m, cfg = _model()
    mb = _batches(cfg)
    total = 0.0
    for ids in mb:
        l = _loss(m(ids), ids) / len(mb)
        l.backward()
        total += float(l)
    ref = {n: p.grad for n, p in m.named_parameters() if p.grad is not None}
    res = run_ranks(_stage, 2)
    assert res[0][2] == (0, 2) and res[1][2] == (2, 4)
    assert res[0][0] is None and abs(res[1][0] - total) < 1e-5
    seen = set()
    for _, grads, _ in res:
        for n, g in grads.items():
            torch.testing.assert_close(g, ref[n], atol=2e-5, rtol=1e-4, msg=n)
            seen.add(n)
    assert "embeddings.embedding.weight" in seen and any(n.startswith("tier1.layers.3") for n in seen)
