"""Function-preserving growth surgery for HLRT (the model-specific half of
progressive growth, ``olympus/core/growth_controller.py`` in the reference,
whose surgery hooks are left abstract there).

Every operation returns a model that computes exactly what the old one did at
the moment of growth, so the loss curve continues where it was; the new
capacity starts contributing as training moves its zero-initialised weights:

* ``widen(factor)``: every dense Tier-1 SwiGLU FFN gets ``d_ff * factor``
  hidden units (rounded up to a multiple of 64).  The new rows of ``W1`` and
  ``W_gate`` are drawn like a fresh layer; the new columns of ``W2`` are zero,
  so the new units add nothing until ``W2`` learns them.
* ``deepen(num_layers, position)``: new Tier-1 blocks are inserted (``"end"``,
  ``"start"`` or a block index) with zero attention-output and FFN-output
  projections, so each new block is the identity on the residual stream.
  PHMA memory reads stay attached to the blocks they followed.
* ``dense_to_moe(num_experts, top_k)``: every dense Tier-1 FFN becomes a
  mixture of ``num_experts`` copies of itself under a freshly initialised
  router; the top-k weights are renormalised to sum to one, so the mixture of
  identical experts equals the dense FFN.

The config (``tier1_d_ff``, ``tier1_num_layers``, ``tier1_moe_*``) is updated
so that checkpoints and later surgery see the grown shapes.  Growth acts on the
plain module; wrap it for sharded training (``wrap_model_fsdp``) afterwards.
"""

from __future__ import annotations

import copy
from typing import Any, Union

import torch
import torch.nn as nn

from olympus.core.growth_controller import GrowthController


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _grow_linear_out(lin: nn.Linear, extra: int, std: float) -> nn.Linear:
    """``lin`` with ``extra`` more output rows, the new rows ~ N(0, std)."""
    new = nn.Linear(lin.in_features, lin.out_features + extra, bias=lin.bias is not None,
                    device=lin.weight.device, dtype=lin.weight.dtype)
    with torch.no_grad():
        new.weight[: lin.out_features].copy_(lin.weight)
        new.weight[lin.out_features:].normal_(0.0, std)
        if lin.bias is not None:
            new.bias[: lin.out_features].copy_(lin.bias)
            new.bias[lin.out_features:].zero_()
    return new


def _grow_linear_in(lin: nn.Linear, extra: int) -> nn.Linear:
    """``lin`` with ``extra`` more input columns, all zero."""
    new = nn.Linear(lin.in_features + extra, lin.out_features, bias=lin.bias is not None,
                    device=lin.weight.device, dtype=lin.weight.dtype)
    with torch.no_grad():
        new.weight.zero_()
        new.weight[:, : lin.in_features].copy_(lin.weight)
        if lin.bias is not None:
            new.bias.copy_(lin.bias)
    return new


def widen_ffn(ffn: nn.Module, d_ff: int, std: float = 0.02) -> None:
    """Grow a :class:`~genesis.model.ffn.SwiGLUFFN` in place to ``d_ff`` hidden units."""
    extra = d_ff - ffn.d_ff
    if extra <= 0:
        return
    ffn.w1 = _grow_linear_out(ffn.w1, extra, std)
    ffn.w_gate = _grow_linear_out(ffn.w_gate, extra, std)
    ffn.w2 = _grow_linear_in(ffn.w2, extra)
    ffn.d_ff = d_ff


def identity_block(template: nn.Module) -> nn.Module:
    """A copy of a Tier-1 block whose output projections are zero: ``x -> x``."""
    blk = copy.deepcopy(template)
    with torch.no_grad():
        for lin in (blk.attn.o_proj, blk.ffn.w2):
            lin.weight.zero_()
            if lin.bias is not None:
                lin.bias.zero_()
    return blk


def dense_to_moe_ffn(ffn: nn.Module, num_experts: int, top_k: int, capacity_factor: float = 1.25) -> nn.Module:
    """A mixture of ``num_experts`` copies of the dense FFN ``ffn`` (same output)."""
    from genesis.model.moe import MoEFFN

    w = ffn.w1.weight
    moe = MoEFFN(d_model=ffn.w1.in_features, d_ff=ffn.d_ff, num_experts=num_experts, top_k=top_k,
                 capacity_factor=capacity_factor).to(device=w.device, dtype=w.dtype)
    for e in moe.experts:
        e.load_state_dict(ffn.state_dict())
    return moe


class HLRTGrowthController(GrowthController):
    """:class:`~olympus.core.growth_controller.GrowthController` with HLRT surgery."""

    def _widen(self, model: nn.Module, factor: float = 2.0, **kwargs: Any) -> nn.Module:
        from genesis.model.ffn import SwiGLUFFN

        layers = model.tier1.layers
        dense = [blk for blk in layers if type(blk.ffn) is SwiGLUFFN]
        if not dense:
            return model
        d_ff = _round_up(int(dense[0].ffn.d_ff * float(factor)), 64)
        for blk in dense:
            widen_ffn(blk.ffn, d_ff)
        model.config.tier1_d_ff = d_ff
        return model

    def _deepen(self, model: nn.Module, num_layers: int = 1, position: Union[str, int] = "end",
                **kwargs: Any) -> nn.Module:
        tier1 = model.tier1
        n = len(tier1.layers)
        if n == 0:
            raise ValueError("deepen needs at least one Tier-1 block to copy the shape from")
        at = n if position == "end" else 0 if position == "start" else int(position)
        if not 0 <= at <= n:
            raise ValueError(f"deepen position {position!r} outside 0..{n}")
        template = tier1.layers[max(at - 1, 0)]
        blocks = list(tier1.layers)
        new = [identity_block(template) for _ in range(int(num_layers))]
        tier1.layers = nn.ModuleList(blocks[:at] + new + blocks[at:])
        if len(tier1.memory_layers):  # memory reads keep following the same blocks
            moved = {}
            for key, layer in tier1.memory_layers.items():
                i = int(key)
                moved[str(i + num_layers if i >= at else i)] = layer
            tier1.memory_layers = nn.ModuleDict(moved)
        model.config.tier1_num_layers = len(tier1.layers)
        return model

    def _dense_to_moe(self, model: nn.Module, num_experts: int = 4, top_k: int = 2, **kwargs: Any) -> nn.Module:
        from genesis.model.ffn import SwiGLUFFN

        cap = float(kwargs.get("capacity_factor", 1.25))
        converted = False
        for blk in model.tier1.layers:
            if type(blk.ffn) is SwiGLUFFN:
                blk.ffn = dense_to_moe_ffn(blk.ffn, num_experts, top_k, cap)
                blk._moe = {"num_experts": num_experts, "top_k": top_k, "capacity_factor": cap}
                converted = True
        if converted:
            model.config.tier1_moe_num_experts = num_experts
            model.config.tier1_moe_top_k = top_k
            model.config.tier1_moe_capacity_factor = cap
        return model
