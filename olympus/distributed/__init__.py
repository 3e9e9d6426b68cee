"""Sharded data parallel training (FSDP-style engine, distributed Muon) and DiLoCo."""
from olympus.distributed.fsdp_wrapper import FSDPConfig, wrap_model_fsdp, get_hlrt_wrap_policy
from olympus.distributed.distributed_orchestrator import DistributedTrainingOrchestrator

__all__ = ["FSDPConfig", "wrap_model_fsdp", "get_hlrt_wrap_policy", "DistributedTrainingOrchestrator"]
