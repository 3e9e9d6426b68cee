"""NVTX ranges around the fused compute+collective paths and the engine's
communication phases, so a timeline (Nsight Systems, or any NVTX consumer)
shows each fused path by name: ``lrb/fsdp/{ag,rs,publish,clip}``,
``lrb/tp/{ag_gemm,gemm_rs}``, ``lrb/ep/{dispatch_push,dispatch_take,
combine_put,combine_pull}``, ``lrb/diloco/outer``.

On by default when CUDA is available (a push/pop pair costs about a
microsecond of host time); ``LRB_NVTX=0`` turns them off."""

from __future__ import annotations

import contextlib
import os

import torch

_ENABLED = os.environ.get("LRB_NVTX", "1") != "0"


def enabled() -> bool:
    return _ENABLED and torch.cuda.is_available()


@contextlib.contextmanager
def nvtx_range(name: str):
    if not enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx_fn(name: str):
    """Decorator form of ``nvtx_range``."""

    def deco(fn):
        import functools

        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            with nvtx_range(name):
                return fn(*args, **kwargs)

        return wrapper

    return deco
