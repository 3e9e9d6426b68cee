from olympus.core.training_context import TrainingContext
from olympus.core.stateful_module import StatefulModule, StateLink
from olympus.core.memory_bus import MemoryBus
from olympus.core.compute_router import ComputeRouter, RoutePlan
from olympus.core.training_orchestrator import TrainingOrchestrator, ModelConfig, ObjectiveConfig
from olympus.core.growth_controller import GrowthController, GrowthEvent

__all__ = [
    "TrainingContext", "StatefulModule", "StateLink", "MemoryBus", "ComputeRouter", "RoutePlan",
    "TrainingOrchestrator", "ModelConfig", "ObjectiveConfig", "GrowthController", "GrowthEvent",
]
