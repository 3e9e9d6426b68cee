"""Configuration loading (``olympus/utils/config.py:18-66``) plus the mapping
of the reference's nested training YAML schema onto :class:`HLRTConfig`.

``load_config(path, overrides)`` returns an OmegaConf ``DictConfig`` when
OmegaConf is installed, else a plain dict; dotted override keys
(``{"model.tier1.layers": 4}``) are applied after loading.

The YAML presets of the reference (``genesis/training/configs/phase*.yaml``)
describe models as ``model.tier1.layers``, ``model.tier2.d_model``,
``model.gate.tier2_threshold`` ... and no code of the reference reads them;
:func:`hlrt_config_from_yaml` does.
"""

from __future__ import annotations

import os
from typing import Any, Dict, Mapping, Optional, Union

try:  # optional, like the reference
    from omegaconf import DictConfig, OmegaConf

    _HAS_OMEGACONF = True
except ImportError:  # pragma: no cover - depends on the environment
    _HAS_OMEGACONF = False


def _apply_overrides(cfg: dict, overrides: Mapping[str, Any]) -> None:
    for key, value in overrides.items():
        node = cfg
        *parents, leaf = key.split(".")
        for p in parents:
            node = node.setdefault(p, {})
        node[leaf] = value


def load_config(path: str, overrides: Optional[Dict[str, Any]] = None) -> Union["DictConfig", Dict[str, Any]]:
    if not os.path.isfile(path):
        raise FileNotFoundError(f"Config file not found: {path}")
    if _HAS_OMEGACONF:
        cfg = OmegaConf.load(path)
        if overrides:
            cfg = OmegaConf.merge(cfg, OmegaConf.create(_nest(overrides)))
        return cfg
    import yaml

    with open(path) as f:
        cfg = yaml.safe_load(f) or {}
    if overrides:
        _apply_overrides(cfg, overrides)
    return cfg


def _nest(flat: Mapping[str, Any]) -> Dict[str, Any]:
    out: Dict[str, Any] = {}
    _apply_overrides(out, flat)
    return out


def _plain(cfg: Any) -> Dict[str, Any]:
    if _HAS_OMEGACONF and isinstance(cfg, DictConfig):
        return OmegaConf.to_container(cfg, resolve=True)  # type: ignore[return-value]
    return dict(cfg)


def hlrt_config_from_yaml(path_or_cfg: Any, overrides: Optional[Dict[str, Any]] = None):
    """Build an :class:`HLRTConfig` from the nested ``model:`` section."""
    from genesis.model.hlrt import HLRTConfig

    cfg = load_config(path_or_cfg, overrides) if isinstance(path_or_cfg, str) else path_or_cfg
    m = _plain(cfg).get("model", {})
    t1, t2, t3, gate = m.get("tier1", {}), m.get("tier2", {}), m.get("tier3", {}), m.get("gate", {})
    kw: Dict[str, Any] = {}

    def put(key: str, value: Any) -> None:
        if value is not None:
            kw[key] = value

    put("vocab_size", m.get("vocab_size"))
    put("d_model", t1.get("d_model"))
    put("tier1_num_layers", t1.get("layers"))
    put("tier1_num_heads", t1.get("heads"))
    put("tier1_num_kv_heads", t1.get("kv_heads"))
    put("tier1_d_ff", t1.get("d_ff"))
    put("tier1_max_seq_len", m.get("max_seq_len"))
    put("tier2_d_model", t2.get("d_model"))
    put("tier2_num_layers", t2.get("layers"))
    put("tier2_num_heads", t2.get("heads"))
    put("tier2_d_ff", t2.get("d_ff"))
    put("num_latent_vectors", t2.get("latent_vectors_per_chunk"))
    put("gate1_chunk_size", t2.get("chunk_size"))
    put("tier2_moe_num_experts", t2.get("moe_num_experts"))
    put("tier2_moe_top_k", t2.get("moe_top_k"))
    put("tier2_max_seq_len", t2.get("max_seq_len"))
    put("tier2_num_kv_heads", t2.get("kv_heads"))
    put("latent_pool_num_heads", t2.get("latent_pool_heads"))
    # extensions of the schema: a Tier-1 mixture of experts and PHMA memory reads
    put("tier1_moe_num_experts", t1.get("moe_num_experts"))
    put("tier1_moe_top_k", t1.get("moe_top_k"))
    put("tier1_moe_d_ff", t1.get("moe_d_ff"))
    put("tier1_moe_shared_experts", t1.get("moe_shared_experts"))
    put("tier1_moe_capacity_factor", t1.get("moe_capacity_factor"))
    mem = m.get("memory", {}) or {}
    put("tier1_memory_every", mem.get("every"))
    put("memory_slots", mem.get("slots"))
    put("memory_top_k", mem.get("top_k"))
    put("tier3_d_model", t3.get("d_model"))
    put("tier3_num_layers", t3.get("layers"))
    put("tier3_num_heads", t3.get("heads"))
    put("tier3_d_ff", t3.get("d_ff"))
    put("tier3_recurrence_steps", t3.get("recurrence_steps"))
    put("tier3_max_seq_len", t3.get("max_seq_len"))
    put("tier3_num_kv_heads", t3.get("kv_heads"))
    put("gate1_threshold", gate.get("tier2_threshold"))
    put("gate2_threshold", gate.get("tier3_threshold"))
    if "dropout" in m:
        for k in ("tier1_dropout", "tier2_dropout", "tier3_dropout"):
            kw[k] = m["dropout"]
    if "rope_base" in m:
        for k in ("tier1_rope_base", "tier2_rope_base", "tier3_rope_base"):
            kw[k] = m["rope_base"]
    if "use_flash_attention" in m:
        for k in ("tier1_use_flash_attention", "tier2_use_flash_attention", "tier3_use_flash_attention"):
            kw[k] = m["use_flash_attention"]
    return HLRTConfig(**kw)


def parse_overrides(items) -> Dict[str, Any]:
    """``["model.tier1.layers=4", "optimizer.muon_lr=0.01"]`` -> dotted-key dict; values
    are parsed as YAML scalars/lists (``4`` -> int, ``[0.9, 0.95]`` -> list, ``true`` -> bool)."""
    import yaml

    out: Dict[str, Any] = {}
    for item in items or ():
        key, sep, value = item.partition("=")
        if not sep or not key:
            raise ValueError(f"override must look like key.path=value, got {item!r}")
        out[key.strip()] = yaml.safe_load(value)
    return out


def trainer_settings_from_yaml(path_or_cfg: Any, overrides: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """The ``optimizer:``, ``scheduler:``, ``training:`` and ``hardware:`` sections of
    the nested schema as the trainer's arguments: ``optimizer_kwargs`` for
    ``MuonAdamWHybrid``, ``scheduler_kwargs`` for ``WSDScheduler`` and the trainer
    ``config`` keys.  Keys absent from the file are absent from the result."""
    cfg = load_config(path_or_cfg, overrides) if isinstance(path_or_cfg, str) else path_or_cfg
    c = _plain(cfg)
    opt, sch, tr, hw = (c.get(k, {}) or {} for k in ("optimizer", "scheduler", "training", "hardware"))
    optimizer: Dict[str, Any] = {}
    scheduler: Dict[str, Any] = {}
    trainer: Dict[str, Any] = {}

    def put(d: Dict[str, Any], key: str, value: Any, conv=None) -> None:
        if value is not None:
            d[key] = conv(value) if conv else value

    put(optimizer, "lr_muon", opt.get("muon_lr"), float)
    put(optimizer, "lr_adamw", opt.get("adamw_lr"), float)
    put(optimizer, "momentum", opt.get("muon_momentum"), float)
    put(optimizer, "betas", opt.get("adamw_betas"), lambda b: tuple(float(x) for x in b))
    put(optimizer, "weight_decay_adamw", opt.get("weight_decay"), float)
    put(optimizer, "ns_steps", opt.get("ns_iterations"), int)
    warm, stable, decay = sch.get("warmup_steps"), sch.get("stable_steps"), sch.get("decay_steps")
    put(scheduler, "base_lr", opt.get("adamw_lr"), float)
    put(scheduler, "min_lr", sch.get("min_lr"), float)
    put(scheduler, "warmup_steps", warm, int)
    put(scheduler, "decay_steps", decay, int)
    if warm is not None and stable is not None:
        scheduler["decay_start"] = int(warm) + int(stable)
        if decay is not None:
            scheduler["total_steps"] = int(warm) + int(stable) + int(decay)
    put(trainer, "batch_size", tr.get("batch_size"), int)
    put(trainer, "gradient_accumulation_steps", tr.get("gradient_accumulation_steps"), int)
    put(trainer, "max_steps", tr.get("max_steps"), int)
    put(trainer, "max_grad_norm", tr.get("gradient_clip"), float)
    put(trainer, "save_interval", tr.get("checkpoint_interval"), int)
    put(trainer, "eval_interval", tr.get("eval_interval"), int)
    put(trainer, "log_interval", tr.get("log_interval"), int)
    put(trainer, "seq_len", tr.get("seq_len", (c.get("data", {}) or {}).get("max_seq_len")), int)
    put(trainer, "device", hw.get("device"))
    put(trainer, "precision", hw.get("precision", tr.get("precision")))
    return {"optimizer_kwargs": optimizer, "scheduler_kwargs": scheduler, "trainer": trainer}
