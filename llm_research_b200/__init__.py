"""B200 (sm_100a) engine of the Olympus/GENESIS framework.

Subpackages:
  ops       -- hot operations (native sm_100a kernels on CUDA, PyTorch oracle on CPU)
  parallel  -- NCCL/NVLink plumbing: FSDP, distributed Muon, TP, EP, DiLoCo, symmetric memory
  models    -- named model presets (the benchmark configurations) and builders
  utils     -- device timing, clock sampling, logging helpers
"""

__version__ = "0.1.0"
