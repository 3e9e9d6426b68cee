"""Causal multi-head / grouped-query attention with RoPE (``genesis/model/attention.py:31-195``).

Parameters and semantics follow the reference: bias-free ``q/k/v/o_proj``,
rotate-half RoPE on q and k at positions ``position_offset ..``, causal mask
aligned to the end of the key sequence (so cached decode works), optional
additive ``attention_mask`` and attention dropout, optional KV cache.

Execution on B200:
  * q, k and v come out of ONE GEMM against the concatenated ``[Wq; Wk; Wv]``;
  * one kernel applies RoPE to q/k and writes them in ``(B, S, H, D)`` layout;
  * attention is the flash-attention kernel with native GQA (K/V heads are
    never repeated in memory) -- the reference materialises the repeated
    K/V (``attention.py:121-126``);
  * the output feeds ``o_proj`` without a transpose copy.
An additive mask or attention dropout (both unsupported by the fused kernel)
takes the explicit ``softmax(QK^T)V`` path, which is what the reference
computes in ``_vanilla_attention``.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from genesis.model.rotary import apply_rotary_emb
from llm_research_b200 import ops
from llm_research_b200.ops.linear import cat_rows, project, qkv_rope

# The reference probes flash-attn here; the fused kernel replaces it.
FLASH_ATTN_AVAILABLE = True


class MultiHeadAttention(nn.Module):
    def __init__(
        self,
        d_model: int,
        num_heads: int,
        num_kv_heads: int | None = None,
        dropout: float = 0.0,
        bias: bool = False,
        use_flash_attention: bool = True,
    ) -> None:
        super().__init__()
        assert d_model % num_heads == 0, "d_model must be divisible by num_heads"
        self.d_model = d_model
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        assert num_heads % self.num_kv_heads == 0, "num_heads must be divisible by num_kv_heads"
        self.head_dim = d_model // num_heads
        self.num_kv_groups = num_heads // self.num_kv_heads
        self.dropout_p = dropout
        self.use_flash_attention = use_flash_attention
        from llm_research_b200.parallel.tp import current_tensor_parallel, mark_tp

        tp = current_tensor_parallel()
        self.tp = tp
        nt = 1 if tp is None else torch.distributed.get_world_size(tp[0])
        if tp is not None:
            assert not bias and num_heads % nt == 0 and self.num_kv_heads % nt == 0, \
                "tensor parallelism splits whole (KV) heads and has no biases"
        # Under tensor parallelism every projection holds this rank's heads only.
        self.q_proj = nn.Linear(d_model, num_heads // nt * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(d_model, self.num_kv_heads // nt * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(d_model, self.num_kv_heads // nt * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(num_heads // nt * self.head_dim, d_model, bias=bias)
        if tp is not None:
            for lin in (self.q_proj, self.k_proj, self.v_proj):
                mark_tp(lin.weight, 0)
            mark_tp(self.o_proj.weight, 1)

    # ------------------------------------------------------------------
    def _qkv(self, x: torch.Tensor) -> torch.Tensor:
        w = cat_rows(self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        b = None
        if self.q_proj.bias is not None:
            b = torch.cat([self.q_proj.bias, self.k_proj.bias, self.v_proj.bias], 0)
        return project(x, w, b)

    def forward_tp(self, x_shard: torch.Tensor, seq_shape, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """Tensor + sequence parallel: ``x_shard`` is this rank's ``(B*S/tp, d)`` rows;
        QKV is an all-gather->GEMM over the group (this rank's heads for all tokens),
        attention runs on the local heads, ``o_proj`` is a GEMM->reduce-scatter back
        to ``(B*S/tp, d)``."""
        from llm_research_b200.parallel.tp import column_parallel, row_parallel

        group, comm = self.tp
        B, S = seq_shape
        nt = torch.distributed.get_world_size(group)
        H, Hkv, D = self.num_heads // nt, self.num_kv_heads // nt, self.head_dim
        w = cat_rows(self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        qkv = column_parallel(x_shard, w, group, comm).view(B, S, -1)
        q, k, v = ops.rope_qkv(qkv, cos, sin, H, Hkv, D, 0)
        drop = self.dropout_p if self.training else 0.0
        if drop == 0.0:
            out = ops.attention(q, k, v, causal=True)
        else:
            qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
            if self.num_kv_groups > 1:
                kh = kh.repeat_interleave(self.num_kv_groups, dim=1)
                vh = vh.repeat_interleave(self.num_kv_groups, dim=1)
            out = self._vanilla_attention(qh, kh, vh, None).transpose(1, 2)
        return row_parallel(out.reshape(B * S, H * D), self.o_proj.weight, group, comm)

    def forward(
        self,
        x: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        attention_mask: Optional[torch.Tensor] = None,
        kv_cache: Optional[object] = None,
        position_offset: int = 0,
    ) -> torch.Tensor:
        if kv_cache is not None and getattr(kv_cache, "is_static", False):
            return self._forward_static(x, cos, sin, kv_cache)
        B, S, _ = x.shape
        H, Hkv, D = self.num_heads, self.num_kv_heads, self.head_dim
        drop = self.dropout_p if self.training else 0.0
        if kv_cache is None and attention_mask is None and drop == 0.0 and self.q_proj.bias is None:
            # one launch: QKV projection with RoPE in the GEMM epilogue (q, k, v are views)
            fused = qkv_rope(x, cat_rows(self.q_proj.weight, self.k_proj.weight, self.v_proj.weight), cos, sin,
                             H, Hkv, D, position_offset)
            if fused is not None:
                out = ops.attention(*fused, causal=True)
                return project(out.reshape(B, S, H * D), self.o_proj.weight, self.o_proj.bias)
        qkv = self._qkv(x)
        # (B,S,H,D) q and (B,S,Hkv,D) k, v with RoPE applied to q and k.
        q, k, v = ops.rope_qkv(qkv, cos, sin, H, Hkv, D, position_offset)
        if kv_cache is None and attention_mask is None and drop == 0.0:
            out = ops.attention(q, k, v, causal=True)
            return project(out.reshape(B, S, H * D), self.o_proj.weight, self.o_proj.bias)

        # General path: cache / additive mask / dropout.
        qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if kv_cache is not None:
            kh, vh = kv_cache.update(kh, vh)
        if attention_mask is None and drop == 0.0:
            out = ops.attention(qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2), causal=True)
            return project(out.reshape(B, S, H * D), self.o_proj.weight, self.o_proj.bias)
        if self.num_kv_groups > 1:
            kh = kh.repeat_interleave(self.num_kv_groups, dim=1)
            vh = vh.repeat_interleave(self.num_kv_groups, dim=1)
        out = self._vanilla_attention(qh, kh, vh, attention_mask)
        return project(out.transpose(1, 2).reshape(B, S, H * D), self.o_proj.weight, self.o_proj.bias)

    def _forward_static(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, cache) -> torch.Tensor:
        """One decode token against a fixed-capacity cache whose position lives on the
        device (``cache.pos``), so the step has the same shapes and the same launches
        every time and can be replayed from a CUDA graph.  ``cos``/``sin`` are the full
        tables; the row of the current position is gathered on the device.  Slots past
        the position are masked; GQA reads the shared K/V heads without repeating them."""
        B, S, _ = x.shape
        H, Hkv, D = self.num_heads, self.num_kv_heads, self.head_dim
        qkv = self._qkv(x)
        q, k, v = ops.rope_qkv(qkv, cos.index_select(0, cache.pos), sin.index_select(0, cache.pos), H, Hkv, D, 0)
        K, V = cache.write(k, v)  # (B, capacity, Hkv, D)
        qg = q.reshape(B, Hkv, H // Hkv, D)
        scores = torch.matmul(qg, K.permute(0, 2, 3, 1)).float() * (1.0 / math.sqrt(D))
        scores = scores.masked_fill(~cache.valid, float("-inf"))
        p = torch.softmax(scores, dim=-1).to(V.dtype)
        out = torch.matmul(p, V.permute(0, 2, 1, 3))  # (B, Hkv, G, D)
        return project(out.reshape(B, 1, H * D), self.o_proj.weight, self.o_proj.bias)

    def _vanilla_attention(
        self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attention_mask: Optional[torch.Tensor] = None
    ) -> torch.Tensor:
        s_q, s_kv = q.size(2), k.size(2)
        scores = torch.matmul(q, k.transpose(-2, -1)) * (1.0 / math.sqrt(self.head_dim))
        causal = torch.full((s_q, s_kv), float("-inf"), device=q.device, dtype=scores.dtype).triu(s_kv - s_q + 1)
        scores = scores + causal
        if attention_mask is not None:
            scores = scores + attention_mask
        probs = F.softmax(scores, dim=-1, dtype=torch.float32).type_as(q)
        probs = F.dropout(probs, p=self.dropout_p, training=self.training)
        return torch.matmul(probs, v)

    def _legacy_rope(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        return apply_rotary_emb(x, cos, sin)
