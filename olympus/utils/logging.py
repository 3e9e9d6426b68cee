"""Logging setup and metric lines (``olympus/utils/logging.py:14-105``).

``setup_logging`` configures a stream handler (and optionally a file) on the
``olympus`` and ``genesis`` loggers; under ``torch.distributed`` only rank 0
logs at INFO unless ``all_ranks``.  ``log_metrics`` writes one
``step=N k=v ...`` line with slash-separated metric names and forwards the
values to wandb when a run is active.
"""

from __future__ import annotations

import logging
import os
import sys
from typing import Any, Dict, Optional

_FMT = "%(asctime)s %(levelname)s [%(name)s] %(message)s"


def _rank() -> int:
    try:
        import torch.distributed as dist

        return dist.get_rank() if dist.is_available() and dist.is_initialized() else int(os.environ.get("RANK", 0))
    except Exception:
        return 0


def setup_logging(level: int = logging.INFO, log_file: Optional[str] = None, use_wandb: bool = False,
                  wandb_project: str = "genesis", wandb_config: Optional[Dict[str, Any]] = None,
                  all_ranks: bool = False) -> logging.Logger:
    rank = _rank()
    eff = level if (all_ranks or rank == 0) else logging.WARNING
    handlers: list = [logging.StreamHandler(sys.stdout)]
    if log_file:
        os.makedirs(os.path.dirname(log_file) or ".", exist_ok=True)
        handlers.append(logging.FileHandler(log_file))
    for name in ("olympus", "genesis", "llm_research_b200"):
        lg = logging.getLogger(name)
        lg.setLevel(eff)
        lg.handlers.clear()
        for h in handlers:
            h.setFormatter(logging.Formatter(f"[rank {rank}] " + _FMT))
            lg.addHandler(h)
        lg.propagate = False
    if use_wandb and rank == 0:
        try:
            import wandb  # type: ignore

            wandb.init(project=wandb_project, config=wandb_config or {})
        except Exception:
            logging.getLogger("olympus").warning("wandb requested but unavailable")
    return logging.getLogger("olympus")


def log_metrics(metrics: Dict[str, Any], step: int, logger: Optional[logging.Logger] = None, prefix: str = "") -> None:
    lg = logger or logging.getLogger("olympus")
    items = {f"{prefix}{k}" if prefix else k: float(v) for k, v in metrics.items()}
    lg.info("step=%d %s", step, " ".join(f"{k}={v:.6g}" for k, v in items.items()))
    try:
        import wandb  # type: ignore

        if wandb.run is not None:
            wandb.log(items, step=step)
    except Exception:
        pass
