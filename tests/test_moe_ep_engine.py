"""An HLRT with a Tier-1 MoE trains through the flat-shard engine with expert
parallelism on gloo CPU ranks: experts are rank-local (not sharded), the rest
is sharded, and local experts are stepped by the optimizer."""

import torch

from tests.dist_utils import run_ranks


def _train(rank, world):
    from genesis.model import HLRT, HLRTConfig
    from llm_research_b200.parallel.expert_parallel import ExpertParallelMoE, expert_parallel
    from llm_research_b200.parallel.fsdp import FlatShardEngine
    from olympus.optim import MuonAdamWHybrid

    torch.manual_seed(0)
    cfg = HLRTConfig(vocab_size=256, d_model=64, tier1_num_layers=2, tier1_num_heads=4, tier1_d_ff=128,
                     gate1_chunk_size=4, num_latent_vectors=2, latent_pool_num_heads=2,
                     tier2_d_model=64, tier2_num_layers=1, tier2_num_heads=4, tier2_d_ff=128,
                     tier3_d_model=64, tier3_num_layers=1, tier3_num_heads=4, tier3_d_ff=128,
                     tier1_moe_num_experts=4, tier1_moe_d_ff=64, tier1_moe_shared_experts=1)
    with expert_parallel(None, None):
        model = HLRT(cfg)
    assert isinstance(model.tier1.layers[0].ffn, ExpertParallelMoE)
    eng = FlatShardEngine(model)
    assert len(eng.local_params) == 2 * cfg.tier1_num_layers
    defaults = MuonAdamWHybrid([torch.nn.Parameter(torch.zeros(2, 2))], lr_muon=0.02, lr_adamw=1e-3).defaults
    opt = eng.make_optimizer(MuonAdamWHybrid, defaults)
    local0 = {n: p.detach().clone() for n, p in eng.local_params}
    g = torch.Generator().manual_seed(rank)
    losses = []
    for _ in range(4):
        ids = torch.randint(0, 256, (2, 32), generator=g)
        out = eng(ids)
        loss = torch.nn.functional.cross_entropy(out["logits"][:, :-1].reshape(-1, 256), ids[:, 1:].reshape(-1))
        (loss + out["aux_loss"]).backward()
        eng.clip_grad_norm_(1.0)
        opt.step()
        opt.zero_grad()
        losses.append(float(loss))
    moved = all(not torch.equal(local0[n], p) for n, p in eng.local_params)
    return losses, moved, eng.full_state_dict()["embeddings.embedding.weight"][:2].clone()


def test_moe_expert_parallel_through_engine():
    res = run_ranks(_train, 2)
    for losses, moved, _ in res:
        assert all(l == l for l in losses) and moved
    torch.testing.assert_close(res[0][2], res[1][2])  # sharded parameters agree across ranks
