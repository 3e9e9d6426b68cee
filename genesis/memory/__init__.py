"""PHMA: working (L1), episodic (L2) and semantic (L3) memory, controller, consistency."""
from genesis.memory.working_memory import WorkingMemory
from genesis.memory.episodic_memory import EpisodicMemory
from genesis.memory.semantic_memory import SemanticMemory
from genesis.memory.memory_controller import MemoryController
from genesis.memory.memory_cross_attention import MemoryCrossAttention
from genesis.memory.memory_consistency import MemoryConsistency

__all__ = ["WorkingMemory", "EpisodicMemory", "SemanticMemory", "MemoryController", "MemoryCrossAttention",
           "MemoryConsistency"]
