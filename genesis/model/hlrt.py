"""HLRT: Hierarchical Latent Reasoning Transformer (``genesis/model/hlrt.py:33-391``).

Forward (training / prefill):

    embed -> Tier 1 -> gate 1 -> [any chunk escalated?]
        yes: latent pooling -> Tier 2 -> plan vector (cached as state)
             -> h += sigmoid(alpha) * plan -> gate 2 -> [any latent escalated?]
                 yes: Tier 3 -> integrate back into the escalated chunks
        no:  h += sigmoid(alpha) * cached plan
    -> RMSNorm -> logits (tied to the embedding unless configured otherwise)

Single-token decode with a KV cache skips the gates and uses the cached plan.
Returns ``{"logits", "hidden_states", "aux_loss"[, "tier_activations"]}``;
``aux_loss = gate_w * (LB(gate1) [+ LB(gate2)]) + moe_w * LB(tier2 MoE)``.

The module tree, parameter names and initialisation (N(0, 0.02) for every
Linear and Embedding weight, zero biases) are those of the reference, so a
checkpoint of either loads into the other and the same seed gives the same
weights.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from genesis.model.conditioning import TopDownConditioning
from genesis.model.embeddings import SharedEmbeddings
from genesis.model.latent_pooling import LatentPooling
from genesis.model.rmsnorm import RMSNorm
from genesis.model.tier1_token_processor import Tier1TokenProcessor
from genesis.model.tier2_semantic_planner import Tier2SemanticPlanner
from genesis.model.tier3_deliberative import Tier3DeliberativeReasoner
from genesis.model.tier_gate import TierGate
from llm_research_b200.ops.linear import dense
from olympus.core.stateful_module import StatefulModule


@dataclass
class HLRTConfig:
    vocab_size: int = 100287
    d_model: int = 1024
    padding_idx: int | None = None
    embedding_dropout: float = 0.0
    tie_word_embeddings: bool = True

    tier1_num_layers: int = 12
    tier1_num_heads: int = 16
    tier1_num_kv_heads: int | None = None
    tier1_d_ff: int | None = None
    tier1_dropout: float = 0.0
    tier1_use_flash_attention: bool = True
    tier1_max_seq_len: int = 8192
    tier1_rope_base: float = 10000.0
    # Tier-1 mixture of experts (an extension: the reference trunk is dense)
    tier1_moe_num_experts: int | None = None
    tier1_moe_top_k: int = 2
    tier1_moe_d_ff: int | None = None
    tier1_moe_shared_experts: int = 0
    tier1_moe_capacity_factor: float = 1.25
    # PHMA semantic-memory reads in the Tier-1 trunk (an extension): after every
    # ``tier1_memory_every``-th block, top-k over a shared bank of ``memory_slots``.
    tier1_memory_every: int = 0
    memory_slots: int = 65536
    memory_top_k: int = 32

    gate1_chunk_size: int = 32
    gate1_threshold: float = 0.5

    num_latent_vectors: int = 8
    latent_pool_num_heads: int = 4
    latent_pool_dropout: float = 0.0

    tier2_d_model: int = 1536
    tier2_num_layers: int = 8
    tier2_num_heads: int = 16
    tier2_num_kv_heads: int | None = None
    tier2_d_ff: int | None = None
    tier2_dropout: float = 0.0
    tier2_use_flash_attention: bool = True
    tier2_max_seq_len: int = 2048
    tier2_rope_base: float = 10000.0
    tier2_moe_num_experts: int | None = None
    tier2_moe_top_k: int = 2

    gate2_chunk_size: int = 1
    gate2_threshold: float = 0.5

    tier3_d_model: int = 1024
    tier3_num_layers: int = 5
    tier3_num_heads: int = 8
    tier3_num_kv_heads: int | None = None
    tier3_d_ff: int | None = None
    tier3_dropout: float = 0.0
    tier3_use_flash_attention: bool = True
    tier3_max_seq_len: int = 1024
    tier3_rope_base: float = 10000.0
    tier3_recurrence_steps: int = 4

    norm_eps: float = 1e-6
    gate_loss_weight: float = 0.01
    moe_loss_weight: float = 0.01

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


class HLRT(StatefulModule):
    def __init__(self, config: HLRTConfig) -> None:
        super().__init__()
        c = config
        self.config = c
        self.embeddings = SharedEmbeddings(c.vocab_size, c.d_model, dropout=c.embedding_dropout, padding_idx=c.padding_idx)
        self.tier1 = Tier1TokenProcessor(
            num_layers=c.tier1_num_layers, d_model=c.d_model, num_heads=c.tier1_num_heads, d_ff=c.tier1_d_ff,
            num_kv_heads=c.tier1_num_kv_heads, dropout=c.tier1_dropout,
            use_flash_attention=c.tier1_use_flash_attention, max_seq_len=c.tier1_max_seq_len,
            rope_base=c.tier1_rope_base, norm_eps=c.norm_eps,
            moe=(dict(num_experts=c.tier1_moe_num_experts, top_k=c.tier1_moe_top_k, d_ff=c.tier1_moe_d_ff,
                      shared=c.tier1_moe_shared_experts, capacity_factor=c.tier1_moe_capacity_factor)
                 if c.tier1_moe_num_experts else None),
            memory=(dict(every=c.tier1_memory_every, d_key=c.d_model, d_value=c.d_model, top_k=c.memory_top_k)
                    if c.tier1_memory_every else None),
        )
        if c.tier1_memory_every:
            from genesis.model.memory_layer import MemoryBank

            self.memory_bank = MemoryBank(c.memory_slots, c.d_model, c.d_model)
            self.tier1.bind_memory(self.memory_bank)
        self.gate1 = TierGate(d_model=c.d_model, chunk_size=c.gate1_chunk_size, threshold=c.gate1_threshold)
        self.latent_pool = LatentPooling(
            input_dim=c.d_model, output_dim=c.tier2_d_model, num_latent_vectors=c.num_latent_vectors,
            num_heads=c.latent_pool_num_heads, chunk_size=c.gate1_chunk_size, dropout=c.latent_pool_dropout,
        )
        self.tier2 = Tier2SemanticPlanner(
            num_layers=c.tier2_num_layers, d_model=c.tier2_d_model, num_heads=c.tier2_num_heads, d_ff=c.tier2_d_ff,
            num_kv_heads=c.tier2_num_kv_heads, dropout=c.tier2_dropout,
            use_flash_attention=c.tier2_use_flash_attention, max_seq_len=c.tier2_max_seq_len,
            rope_base=c.tier2_rope_base, norm_eps=c.norm_eps,
            moe_num_experts=c.tier2_moe_num_experts, moe_top_k=c.tier2_moe_top_k,
        )
        self.gate2 = TierGate(d_model=c.tier2_d_model, chunk_size=c.gate2_chunk_size, threshold=c.gate2_threshold)
        self.tier3 = Tier3DeliberativeReasoner(
            num_layers=c.tier3_num_layers, input_dim=c.tier2_d_model, d_model=c.tier3_d_model,
            num_heads=c.tier3_num_heads, d_ff=c.tier3_d_ff, num_kv_heads=c.tier3_num_kv_heads,
            dropout=c.tier3_dropout, use_flash_attention=c.tier3_use_flash_attention,
            max_seq_len=c.tier3_max_seq_len, rope_base=c.tier3_rope_base, norm_eps=c.norm_eps,
            recurrence_steps=c.tier3_recurrence_steps,
        )
        self.conditioning = TopDownConditioning(d_model=c.d_model, tier2_dim=c.tier2_d_model, chunk_size=c.gate1_chunk_size)
        self.output_norm = RMSNorm(c.d_model, eps=c.norm_eps)
        self.output_proj = None if c.tie_word_embeddings else nn.Linear(c.d_model, c.vocab_size, bias=False)
        # built under a tensor-parallel context: the fused head + loss splits the vocabulary
        # over that group (head weights stay replicated, the gradients come back replicated)
        from llm_research_b200.parallel.tp import enclosing_tensor_parallel_group

        self._vocab_parallel_group = enclosing_tensor_parallel_group()
        self.register_state("last_plan_vector", torch.zeros(1, c.d_model), persistent=False)
        self._init_weights()

    def _init_weights(self) -> None:
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)

    # ------------------------------------------------------------------
    def _cached_plan(self, batch: int) -> torch.Tensor:
        plan = self.link_state("last_plan_vector")
        if plan.shape[0] == 1 and batch > 1:
            plan = plan.expand(batch, -1)
        elif plan.shape[0] != batch:
            plan = plan[:1].expand(batch, -1)
        return plan

    # ------------------------------------------------------------------
    # Escalation without host reads.  The reference decides on the host whether
    # any chunk escalates (``bool(mask.any())``) and sizes the latent buffer by the
    # largest per-sample count (another host read).  Here Tiers 2/3 always run on a
    # buffer of all C chunk slots and the decisions are device-side selects:
    #   * slots past the reference's count n (a device scalar) hold zero latents and
    #     come after every real slot, so the causal Tier-2/3 transformers leave the
    #     first n slots exactly as the reference computes them;
    #   * the plan averages the first n slots and the Tier-2 gate's balance loss
    #     counts the first n * L latent positions only;
    #   * "nothing escalated" selects the cached-plan path with torch.where (the
    #     other branch gets zero gradient), and the stored plan is updated only
    #     when something escalated.
    # Tier-2 MoE balances its router over every token it sees, so with a Tier-2
    # MoE the reference path (with its host reads) is kept.
    fixed_escalation = True

    def _fixed_escalation(self) -> bool:
        return self.fixed_escalation and not self.config.tier2_moe_num_experts

    def _escalate_fixed(self, t1, g1_mask, sel1, acts, keep_acts):
        B = t1.shape[0]
        L = self.config.num_latent_vectors
        any1 = sel1.any()
        latents, n1 = self.latent_pool.forward_fixed(t1, g1_mask)
        if keep_acts:
            acts["latent_vectors"] = latents
        t2 = self.tier2(latents)
        if keep_acts:
            acts["tier2"] = t2
        plan = self.conditioning.compute_plan_vector(t2, n1)
        cached = self._cached_plan(B)
        old = self.get_state("last_plan_vector")
        new = plan.detach().mean(dim=0, keepdim=True).to(old.dtype)
        self.set_state("last_plan_vector", torch.where(any1, new, old))
        t1_plan = self.conditioning.apply_cached_plan(t1, plan)

        g2_mask, g2_scores = self.gate2(t2.reshape(B, -1, self.config.tier2_d_model))
        if keep_acts:
            acts["gate2_scores"] = g2_scores
        aux = self.config.gate_loss_weight * self.gate2.load_balance_loss(valid_len=n1 * L)
        sel2 = g2_mask if g2_mask.dtype == torch.bool else g2_mask > 0.5
        live = torch.arange(sel2.shape[1], device=sel2.device) < n1 * L
        any2 = (sel2 & live).any()
        t3 = self.tier3(t2)
        if keep_acts:
            acts["tier3"] = t3
        t1_t3 = self.conditioning.integrate_tier3(t1_plan, t3, g1_mask, g2_mask, fixed=True)
        t1_esc = torch.where(any2, t1_t3, t1_plan)
        t1_out = torch.where(any1, t1_esc, self.conditioning.apply_cached_plan(t1, cached))
        return t1_out, aux * any1.to(aux.dtype)

    def _head(self, h: torch.Tensor) -> torch.Tensor:
        w = self.output_proj.weight if self.output_proj is not None else self.embeddings.weight
        return dense(h, w)

    def forward(
        self,
        input_ids: torch.Tensor,
        attention_mask: Optional[torch.Tensor] = None,
        return_tier_activations: bool = False,
        kv_cache: Optional[Any] = None,
        position_offset: int = 0,
        labels: Optional[torch.Tensor] = None,
    ) -> Dict[str, Any]:
        """``labels`` (an extension; per-position targets, ``-100`` ignored): the
        head and the token cross-entropy run chunk by chunk
        (``llm_research_b200.ops.loss.linear_cross_entropy``) and the output
        carries ``lm_loss`` instead of the ``(B, S, vocab)`` logits."""
        x = self.embeddings(input_ids)
        t1 = self.tier1(x, attention_mask=attention_mask, kv_cache=kv_cache, position_offset=position_offset)
        return self.forward_after_tier1(t1, attention_mask=attention_mask,
                                        return_tier_activations=return_tier_activations, kv_cache=kv_cache,
                                        labels=labels)

    def forward_after_tier1(
        self,
        t1: torch.Tensor,
        attention_mask: Optional[torch.Tensor] = None,
        return_tier_activations: bool = False,
        kv_cache: Optional[Any] = None,
        labels: Optional[torch.Tensor] = None,
    ) -> Dict[str, Any]:
        """Everything after the Tier-1 trunk: gates, Tiers 2/3, plan conditioning and
        the head (the last pipeline stage runs this on the trunk's output)."""
        B, S = t1.shape[0], t1.shape[1]
        acts: Dict[str, Any] = {}
        if return_tier_activations:
            acts["tier1"] = t1

        if kv_cache is not None and S == 1:
            t1 = self.conditioning.apply_cached_plan(t1, self._cached_plan(B))
            h = self.output_norm(t1)
            out: Dict[str, Any] = {
                "logits": self._head(h),
                "hidden_states": h,
                "aux_loss": torch.zeros((), device=t1.device),  # filled on the device (graph-capturable)
            }
            if return_tier_activations:
                out["tier_activations"] = acts
            return out

        g1_mask, g1_scores = self.gate1(t1)
        if return_tier_activations:
            acts["gate1_scores"] = g1_scores
        sel1 = g1_mask if g1_mask.dtype == torch.bool else g1_mask > 0.5
        aux = self.config.gate_loss_weight * self.gate1.load_balance_loss()
        if self.config.tier1_moe_num_experts:
            for layer in self.tier1.layers:
                aux = aux + self.config.moe_loss_weight * layer.ffn.load_balance_loss().to(aux.device)

        if self._fixed_escalation():
            t1, aux_esc = self._escalate_fixed(t1, g1_mask, sel1, acts, return_tier_activations)
            aux = aux + aux_esc
        elif bool(sel1.any()):
            latents = self.latent_pool(t1, g1_mask)
            if return_tier_activations:
                acts["latent_vectors"] = latents
            t2 = self.tier2(latents)
            if return_tier_activations:
                acts["tier2"] = t2
            aux = aux + self.config.moe_loss_weight * self.tier2.load_balance_loss().to(aux.device)
            plan = self.conditioning.compute_plan_vector(t2)
            self.set_state("last_plan_vector", plan.detach().mean(dim=0, keepdim=True))
            t1 = self.conditioning.apply_cached_plan(t1, plan)

            g2_mask, g2_scores = self.gate2(t2.reshape(B, -1, self.config.tier2_d_model))
            if return_tier_activations:
                acts["gate2_scores"] = g2_scores
            aux = aux + self.config.gate_loss_weight * self.gate2.load_balance_loss()
            sel2 = g2_mask if g2_mask.dtype == torch.bool else g2_mask > 0.5
            if bool(sel2.any()):
                t3 = self.tier3(t2)
                if return_tier_activations:
                    acts["tier3"] = t3
                t1 = self.conditioning.integrate_tier3(t1, t3, g1_mask, g2_mask)
        else:
            t1 = self.conditioning.apply_cached_plan(t1, self._cached_plan(B))

        h = self.output_norm(t1)
        if labels is not None:
            from llm_research_b200.ops.loss import linear_cross_entropy, vocab_parallel_linear_cross_entropy

            w = self.output_proj.weight if self.output_proj is not None else self.embeddings.weight
            if self._vocab_parallel_group is not None:
                lm_loss = vocab_parallel_linear_cross_entropy(h, w, labels, self._vocab_parallel_group)
            else:
                lm_loss = linear_cross_entropy(h, w, labels)
            out = {"logits": None, "lm_loss": lm_loss, "hidden_states": h, "aux_loss": aux}
        else:
            out = {"logits": self._head(h), "hidden_states": h, "aux_loss": aux}
        if return_tier_activations:
            out["tier_activations"] = acts
        return out
