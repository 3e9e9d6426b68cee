"""Utilities: configuration, metrics, seeding, checkpointing, logging, profiling."""
from olympus.utils.config import load_config, hlrt_config_from_yaml
from olympus.utils.metrics import MetricsAggregator
from olympus.utils.seeds import set_seed
from olympus.utils.checkpointing import CheckpointManager
from olympus.utils.logging import setup_logging, log_metrics
from olympus.utils.profiling import DeviceTimer, MemoryTracker, count_parameters, get_gpu_memory_stats

__all__ = ["load_config", "hlrt_config_from_yaml", "MetricsAggregator", "set_seed", "CheckpointManager",
           "setup_logging", "log_metrics", "DeviceTimer", "MemoryTracker", "count_parameters", "get_gpu_memory_stats"]
