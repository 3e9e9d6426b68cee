"""Tier 1: the pre-norm transformer trunk over the full token sequence
(``genesis/model/tier1_token_processor.py:22-169``).

Block: ``x += attn(RMSNorm(x)); x += ffn(RMSNorm(x))``.  The second residual
add is fused with the FFN RMSNorm (one kernel reads ``x`` and the attention
output once and writes both the new residual stream and its norm).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from genesis.model.attention import MultiHeadAttention
from genesis.model.ffn import SwiGLUFFN
from genesis.model.rmsnorm import RMSNorm
from genesis.model.rotary import RotaryEmbedding


class TransformerBlock(nn.Module):
    def __init__(
        self,
        d_model: int,
        num_heads: int,
        d_ff: int | None = None,
        num_kv_heads: int | None = None,
        dropout: float = 0.0,
        use_flash_attention: bool = True,
        norm_eps: float = 1e-6,
        moe: Optional[dict] = None,
    ) -> None:
        super().__init__()
        self._moe = moe
        self.attn_norm = RMSNorm(d_model, eps=norm_eps)
        self.attn = MultiHeadAttention(
            d_model=d_model, num_heads=num_heads, num_kv_heads=num_kv_heads,
            dropout=dropout, use_flash_attention=use_flash_attention,
        )
        self.ffn_norm = RMSNorm(d_model, eps=norm_eps)
        self.ffn = self._make_ffn(d_model, d_ff, dropout)

    def _make_ffn(self, d_model: int, d_ff: int | None, dropout: float) -> nn.Module:
        moe = getattr(self, "_moe", None)
        if moe:
            from genesis.model.moe import MoEFFN
            from llm_research_b200.parallel.expert_parallel import ExpertParallelMoE, current_expert_parallel

            ep = current_expert_parallel()
            if ep is not None:  # this rank's experts only
                return ExpertParallelMoE(d_model, moe.get("d_ff") or d_ff, moe["num_experts"], top_k=moe.get("top_k", 2),
                                         capacity_factor=moe.get("capacity_factor", 1.25), group=ep[0],
                                         shared_expert=moe.get("shared", 0) > 0, comm=ep[1])

            return MoEFFN(d_model=d_model, d_ff=moe.get("d_ff") or d_ff, num_experts=moe["num_experts"],
                          top_k=moe.get("top_k", 2), capacity_factor=moe.get("capacity_factor", 1.25),
                          dropout=dropout, enforce_capacity=True, num_shared_experts=moe.get("shared", 0))
        return SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout)

    def forward(
        self,
        x: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        attention_mask: Optional[torch.Tensor] = None,
        kv_cache: Optional[object] = None,
        position_offset: int = 0,
        seq_shape: Optional[tuple] = None,
    ) -> torch.Tensor:
        if seq_shape is not None:  # tensor + sequence parallel: x is this rank's (B*S/tp, d) rows
            return self._forward_tp(x, cos, sin, seq_shape)
        h = self.attn(self.attn_norm(x), cos, sin, attention_mask=attention_mask,
                      kv_cache=kv_cache, position_offset=position_offset)
        normed, x = self.ffn_norm.forward_residual(h, x)
        if isinstance(self.ffn, SwiGLUFFN):
            return self.ffn(normed, residual=x)  # the residual added in the down projection's epilogue
        return x + self.ffn(normed)

    def _forward_tp(self, x, cos, sin, seq_shape):
        from llm_research_b200 import ops
        from llm_research_b200.parallel.tp import sum_grad

        group = self.attn.tp[0]
        # The norms see this rank's tokens only: their weight gradients are summed over the group.
        h = self.attn.forward_tp(ops.rms_norm(x, sum_grad(self.attn_norm.weight, group), self.attn_norm.eps),
                                 seq_shape, cos, sin)
        normed, x = ops.rms_norm_residual(h, x, sum_grad(self.ffn_norm.weight, group), self.ffn_norm.eps)
        return x + self.ffn.forward_tp(normed)


class Tier1TokenProcessor(nn.Module):
    def __init__(
        self,
        num_layers: int,
        d_model: int,
        num_heads: int,
        d_ff: int | None = None,
        num_kv_heads: int | None = None,
        dropout: float = 0.0,
        use_flash_attention: bool = True,
        max_seq_len: int = 8192,
        rope_base: float = 10000.0,
        norm_eps: float = 1e-6,
        moe: Optional[dict] = None,
        memory: Optional[dict] = None,
    ) -> None:
        super().__init__()
        self.rotary_emb = RotaryEmbedding(dim=d_model // num_heads, max_seq_len=max_seq_len, base=rope_base)
        from llm_research_b200.parallel.tp import tensor_parallel_scope

        with tensor_parallel_scope():  # blocks split only under an enclosing ``tensor_parallel`` context
            self.layers = nn.ModuleList([
                TransformerBlock(
                    d_model=d_model, num_heads=num_heads, d_ff=d_ff, num_kv_heads=num_kv_heads,
                    dropout=dropout, use_flash_attention=use_flash_attention, norm_eps=norm_eps, moe=moe,
                )
                for _ in range(num_layers)
            ])
            # PHMA memory reads after every ``memory["every"]``-th block (extension).
            self.memory_layers = nn.ModuleDict()
            if memory and memory.get("every"):
                from genesis.model.memory_layer import MemoryReadLayer

                for i in range(num_layers):
                    if (i + 1) % memory["every"] == 0:
                        self.memory_layers[str(i)] = MemoryReadLayer(
                            d_model, memory["d_key"], memory["d_value"], top_k=memory.get("top_k", 32),
                            norm_eps=norm_eps)

    def bind_memory(self, bank) -> None:
        for m in self.memory_layers.values():
            m.bind(bank)

    def forward(
        self,
        x: torch.Tensor,
        attention_mask: Optional[torch.Tensor] = None,
        kv_cache: Optional[object] = None,
        position_offset: int = 0,
        layer_range: Optional[tuple] = None,
    ) -> torch.Tensor:
        """``layer_range = (start, end)`` runs blocks ``start .. end-1`` only (a pipeline
        stage); the memory read after a block belongs to that block's stage."""
        cos, sin = self.rotary_emb(position_offset + x.size(1))
        if layer_range is not None:
            start, end = layer_range
            for i in range(start, end):
                x = self.layers[i](x, cos, sin, attention_mask=attention_mask, position_offset=position_offset)
                if str(i) in self.memory_layers:
                    x = self.memory_layers[str(i)](x)
            return x
        tp = self.layers[0].attn.tp if len(self.layers) else None
        if tp is not None and kv_cache is None and attention_mask is None and position_offset == 0:
            from llm_research_b200.parallel.tp import gather_sequence, scatter_sequence

            B, S, d = x.shape
            h = scatter_sequence(x, tp[0])
            for i, layer in enumerate(self.layers):
                h = layer(h, cos, sin, seq_shape=(B, S))
                if str(i) in self.memory_layers:
                    h = self.memory_layers[str(i)](h)
            return gather_sequence(h, tp[0], (B, S, d))
        assert tp is None, "tensor-parallel Tier 1 runs full causal sequences (no cache / mask / offset)"
        for i, layer in enumerate(self.layers):
            x = layer(x, cos, sin, attention_mask=attention_mask,
                      kv_cache=kv_cache[i] if kv_cache is not None else None,
                      position_offset=position_offset)
            if str(i) in self.memory_layers:
                x = self.memory_layers[str(i)](x)
        return x
