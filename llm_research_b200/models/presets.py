"""Named model configurations.

``genesis-1b``  -- the 24-layer dense trunk (d_model 2048, 16 heads, SwiGLU
                   ffn 5632, vocab 32000, RoPE) as HLRT Tier 1.  Tiers 2 and 3
                   carry no transformer layers, so the layer count and the
                   FLOPs are those of the named dense model; the hierarchy
                   (gate, latent pooling, plan conditioning, Tier-3
                   projections and integration) still runs every step.
``genesis-7b``  -- 32 layers, d_model 4096, 32 query / 8 KV heads, ffn 11008,
                   vocab 32000, same tier layout, and a PHMA semantic-memory
                   read after every 4th block (65536 slots x 4096, top-32).
``genesis-7b-nomem`` -- the same trunk without the memory reads.
``genesis-7b-nvfp4`` -- genesis-7b, trained with NVFP4 linears (set by the
                   trainer / bench with ``--precision nvfp4``).
``genesis-40b-moe`` -- 32 layers, d_model 4096, 32 / 8 heads, vocab 32000,
                   every Tier-1 FFN a mixture of 16 routed SwiGLU experts
                   (ffn 6144, top-2 softmax routing, capacity 1.25) plus one
                   shared expert: ~42B parameters, ~8.6B active per token.
``genesis-40b-moe-2l`` -- two layers of genesis-40b-moe, for quick checks.
``tiny``        -- the CPU plumbing configuration: vocab 32000, d_model 256,
                   every tier 4 layers / 4 heads / ffn 1024, Tier-3
                   recurrence 2, a PHMA read of 1024 slots x 256 (top-8)
                   after the 4th block.
``toy``         -- a few-hundred-thousand-parameter model for smoke tests.
"""

from __future__ import annotations

from typing import Callable, Dict

from genesis.model.hlrt import HLRTConfig


def _trunk(vocab: int, d: int, layers: int, heads: int, kv_heads: int | None, ffn: int, seq: int) -> HLRTConfig:
    return HLRTConfig(
        vocab_size=vocab,
        d_model=d,
        tier1_num_layers=layers,
        tier1_num_heads=heads,
        tier1_num_kv_heads=kv_heads,
        tier1_d_ff=ffn,
        tier1_max_seq_len=seq,
        gate1_chunk_size=32,
        num_latent_vectors=8,
        latent_pool_num_heads=heads,
        tier2_d_model=d,
        tier2_num_layers=0,
        tier2_num_heads=heads,
        tier2_max_seq_len=max(seq // 4, 256),
        tier3_d_model=d,
        tier3_num_layers=0,
        tier3_num_heads=heads,
        tier3_max_seq_len=max(seq // 4, 256),
        tier3_recurrence_steps=1,
    )


def _moe_trunk(c: HLRTConfig, experts: int, top_k: int, d_ff: int, shared: int, cap: float) -> HLRTConfig:
    c.tier1_moe_num_experts = experts
    c.tier1_moe_top_k = top_k
    c.tier1_moe_d_ff = d_ff
    c.tier1_moe_shared_experts = shared
    c.tier1_moe_capacity_factor = cap
    return c


def _phma(c: HLRTConfig, every: int = 4, slots: int = 65536, top_k: int = 32) -> HLRTConfig:
    c.tier1_memory_every = every
    c.memory_slots = slots
    c.memory_top_k = top_k
    return c


PRESETS: Dict[str, Callable[[], HLRTConfig]] = {
    "genesis-1b": lambda: _trunk(32000, 2048, 24, 16, None, 5632, 4096),
    "genesis-7b": lambda: _phma(_trunk(32000, 4096, 32, 32, 8, 11008, 4096)),
    "genesis-7b-nvfp4": lambda: _phma(_trunk(32000, 4096, 32, 32, 8, 11008, 4096)),
    # the dense 7B trunk without the memory reads
    "genesis-7b-nomem": lambda: _trunk(32000, 4096, 32, 32, 8, 11008, 4096),
    "genesis-40b-moe": lambda: _moe_trunk(_trunk(32000, 4096, 32, 32, 8, 6144, 4096), 16, 2, 6144, 1, 1.25),
    # two layers of genesis-40b-moe (same layer shapes), for quick multi-GPU checks
    "genesis-40b-moe-2l": lambda: _moe_trunk(_trunk(32000, 4096, 2, 32, 8, 6144, 4096), 16, 2, 6144, 1, 1.25),
    "tiny": lambda: _phma(HLRTConfig(
        vocab_size=32000, d_model=256,
        tier1_num_layers=4, tier1_num_heads=4, tier1_d_ff=1024,
        tier2_d_model=256, tier2_num_layers=4, tier2_num_heads=4, tier2_d_ff=1024,
        tier3_d_model=256, tier3_num_layers=4, tier3_num_heads=4, tier3_d_ff=1024,
        tier3_recurrence_steps=2, latent_pool_num_heads=4,
    ), every=4, slots=1024, top_k=8),
    "toy": lambda: HLRTConfig(
        vocab_size=512, d_model=128, tier1_num_layers=2, tier1_num_heads=2, tier1_d_ff=256,
        gate1_chunk_size=16, num_latent_vectors=4, latent_pool_num_heads=2,
        tier2_d_model=128, tier2_num_layers=1, tier2_num_heads=2, tier2_d_ff=256,
        tier3_d_model=128, tier3_num_layers=1, tier3_num_heads=2, tier3_d_ff=256, tier3_recurrence_steps=2,
    ),
}


def build_hlrt_config(name: str) -> HLRTConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    return PRESETS[name]()


def count_flops_per_token(cfg: HLRTConfig, seq_len: int) -> float:
    """Training FLOPs per token of the Tier-1 trunk + head (6N + causal attention)."""
    d, L = cfg.d_model, cfg.tier1_num_layers
    hkv = cfg.tier1_num_kv_heads or cfg.tier1_num_heads
    hd = d // cfg.tier1_num_heads
    ffn = cfg.tier1_d_ff or ((int(8 / 3 * d) + 255) // 256) * 256
    per_layer = d * d * 2 + 2 * d * hkv * hd + 3 * d * ffn
    if cfg.tier1_moe_num_experts:  # active parameters: top-k routed + shared experts, and the router
        mff = cfg.tier1_moe_d_ff or ffn
        per_layer = (d * d * 2 + 2 * d * hkv * hd + 3 * d * mff * (cfg.tier1_moe_top_k + cfg.tier1_moe_shared_experts)
                     + d * cfg.tier1_moe_num_experts)
    matmul_params = L * per_layer + cfg.vocab_size * d
    attn = L * 2 * 2 * seq_len * d / 2  # QK^T and PV, causal half, per token (fwd)
    mem = 0.0
    if cfg.tier1_memory_every:  # q / value / gate projections (trained) + the bank similarity (forward only)
        n_mem = L // cfg.tier1_memory_every
        mem = n_mem * (6.0 * 4 * d * d + 2.0 * cfg.memory_slots * d)
    return 6.0 * matmul_params + 3.0 * attn + mem
