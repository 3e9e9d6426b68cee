"""Fully-sharded wrapping of GENESIS models (``olympus/distributed/fsdp_wrapper.py:31-200``).

:func:`wrap_model_fsdp` returns a
:class:`~llm_research_b200.parallel.fsdp.FlatShardEngine` configured from an
:class:`FSDPConfig`:

* ``sharding_strategy``: ``FULL_SHARD`` (ZeRO-3: parameters re-gathered for
  the backward), ``SHARD_GRAD_OP`` (ZeRO-2: gathered once per micro-step),
  ``NO_SHARD`` (DDP-like: every rank holds the whole model and optimizer,
  unit gradients are averaged with an all-reduce), ``HYBRID_SHARD`` (sharded
  within a node, replicated across nodes; on a single node it is
  ``FULL_SHARD``, and a group spanning several nodes is rejected);
* ``mixed_precision``: ``bf16``/``fp16`` compute copies (fp32 master weights
  and fp32 gradient accumulation always), ``fp32`` computes in fp32;
* ``activation_checkpointing``: per-transformer-block recomputation (the
  reference's version is a no-op because it imports a module that does not
  exist, ``fsdp_wrapper.py:105-110``);
* ``backward_prefetch``: the engine always prefetches one unit ahead.

Sharding units are the Tier-1 transformer blocks; the reference wraps whole
tiers (``get_hlrt_wrap_policy``), which gathers an entire tier at once.
"""

from __future__ import annotations

import functools
import logging
from dataclasses import dataclass
from typing import Any, Optional, Set, Type

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)

_STRATEGIES = ("FULL_SHARD", "SHARD_GRAD_OP", "NO_SHARD", "HYBRID_SHARD")


@dataclass
class FSDPConfig:
    sharding_strategy: str = "FULL_SHARD"
    mixed_precision: str = "bf16"
    activation_checkpointing: bool = True
    cpu_offload: bool = False
    backward_prefetch: str = "BACKWARD_PRE"
    min_num_params: int = 1_000_000
    # Extensions (not in the reference): shard over this group instead of the
    # world; ``tp_group`` is the tensor-parallel group of the Tier-1 trunk.
    process_group: Any = None
    tp_group: Any = None


def get_sharding_strategy(name: str) -> str:
    if name not in _STRATEGIES:
        raise ValueError(f"Unknown sharding strategy: {name}. Options: {list(_STRATEGIES)}")
    return name


def get_mixed_precision(name: Optional[str]) -> Optional[torch.dtype]:
    if name == "bf16":
        return torch.bfloat16
    if name == "fp16":
        return torch.float16
    if name in ("fp32", "none", None):
        return None
    raise ValueError(f"Unknown precision: {name}. Options: bf16, fp16, fp32")


def get_backward_prefetch(name: str) -> Optional[str]:
    return {"BACKWARD_PRE": "BACKWARD_PRE", "BACKWARD_POST": "BACKWARD_POST", "none": None}.get(name)


def get_hlrt_wrap_policy(min_num_params: int = 1_000_000):
    """Return the set of module classes that become sharding units."""
    from genesis.model.tier1_token_processor import TransformerBlock

    classes: Set[Type[nn.Module]] = {TransformerBlock}
    return functools.partial(lambda module, classes=classes: type(module) in classes)


def wrap_model_fsdp(model: nn.Module, fsdp_config: FSDPConfig, device_id: Optional[int] = None):
    from genesis.model.memory_layer import MemoryReadLayer
    from genesis.model.tier1_token_processor import TransformerBlock
    from llm_research_b200.parallel.fsdp import FlatShardEngine

    strategy = get_sharding_strategy(fsdp_config.sharding_strategy)
    dtype = get_mixed_precision(fsdp_config.mixed_precision) or torch.float32
    device = torch.device("cuda", device_id) if device_id is not None and torch.cuda.is_available() else next(model.parameters()).device
    if strategy == "HYBRID_SHARD" and torch.distributed.is_initialized():
        from llm_research_b200.parallel.symm import single_node

        if not single_node(fsdp_config.process_group):
            raise NotImplementedError("HYBRID_SHARD across several nodes (shard within a node, replicate across "
                                      "nodes) is not supported; use FULL_SHARD or NO_SHARD")
    if fsdp_config.activation_checkpointing:
        apply_activation_checkpointing(model)
    engine = FlatShardEngine(
        model,
        compute_dtype=dtype,
        reshard_after_forward=(strategy in ("FULL_SHARD", "HYBRID_SHARD")),
        replicate=(strategy == "NO_SHARD"),
        unit_classes=(TransformerBlock, MemoryReadLayer),
        device=device,
        process_group=fsdp_config.process_group,
        tp_group=fsdp_config.tp_group,
    )
    logger.info("wrapped %s: %s, compute %s, %.1fM params", type(model).__name__, strategy, dtype,
                sum(p.numel for p in engine.params) / 1e6)
    return engine


def apply_activation_checkpointing(model: nn.Module) -> None:
    """Recompute every Tier-1 transformer block in the backward pass."""
    from genesis.model.tier1_token_processor import TransformerBlock
    from torch.nn.utils.stateless import _reparametrize_module
    from torch.utils.checkpoint import checkpoint

    for m in model.modules():
        if type(m) is TransformerBlock and not getattr(m, "_lrb_ckpt", False):
            inner = m.forward

            def fwd(*args, _inner=inner, _m=m, **kwargs):
                if not (torch.is_grad_enabled() and kwargs.get("kv_cache") is None):
                    return _inner(*args, **kwargs)
                # The recomputation runs after any functional_call context has
                # exited; re-bind the exact weight tensors of this forward.
                snap = dict(_m.named_parameters())

                def run(*a):
                    with _reparametrize_module(_m, snap):
                        return _inner(*a, **kwargs)

                return checkpoint(run, *args, use_reentrant=False)

            m.forward = fwd
            m._lrb_ckpt = True
