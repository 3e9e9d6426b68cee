"""Interval checkpointing with rotation (``olympus/utils/checkpointing.py:16-166``).

Files ``{prefix}_step{step:08d}.pt`` hold ``{"step", "model_state_dict",
"optimizer_state_dict", **extra}``; at most ``max_to_keep`` are kept.

Differences from the reference:
* ``load`` recognises both layouts of ``model_state_dict`` -- with the
  ``_olympus_*`` extras written by ``StatefulModule.state_dict_with_state``
  and without.  The reference checks a key that is never written
  (``__stateful_states__``, ``checkpointing.py:138``) and then fails the strict
  load on the extras.
* ``async_save=True`` copies the tensors to host memory on the caller's
  thread and writes the file on a background thread, so the GPU step does not
  wait for the file system; ``wait()`` joins the pending write.
"""

from __future__ import annotations

import glob
import logging
import os
import threading
from typing import Any, Dict, List, Optional

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)


def _to_cpu(obj: Any) -> Any:
    if isinstance(obj, torch.Tensor):
        return obj.detach().to("cpu", copy=True)
    if isinstance(obj, dict):
        return {k: _to_cpu(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_cpu(v) for v in obj)
    return obj


class CheckpointManager:
    def __init__(self, save_dir: str, save_interval: int = 1000, max_to_keep: int = 5, prefix: str = "ckpt",
                 async_save: bool = False) -> None:
        self.save_dir = save_dir
        self.save_interval = save_interval
        self.max_to_keep = max_to_keep
        self.prefix = prefix
        self.async_save = async_save
        os.makedirs(save_dir, exist_ok=True)
        self._saved: List[str] = []
        self._pending: Optional[threading.Thread] = None

    def _path(self, step: int) -> str:
        return os.path.join(self.save_dir, f"{self.prefix}_step{step:08d}.pt")

    def maybe_save(self, step: int, model: nn.Module, optimizer: torch.optim.Optimizer,
                   extra: Optional[Dict[str, Any]] = None, force: bool = False) -> Optional[str]:
        if not force and step % self.save_interval != 0:
            return None
        from olympus.core.stateful_module import StatefulModule

        state: Dict[str, Any] = {
            "step": step,
            "model_state_dict": model.state_dict_with_state() if isinstance(model, StatefulModule) else model.state_dict(),
            "optimizer_state_dict": optimizer.state_dict(),
        }
        if extra:
            state.update(extra)
        path = self._path(step)
        if self.async_save:
            self.wait()
            host = _to_cpu(state)
            self._pending = threading.Thread(target=self._write, args=(host, path), daemon=True)
            self._pending.start()
        else:
            self._write(state, path)
        return path

    def _write(self, state: Dict[str, Any], path: str) -> None:
        tmp = path + ".tmp"
        torch.save(state, tmp)
        os.replace(tmp, path)  # a crash mid-write never leaves a truncated checkpoint
        self._saved.append(path)
        logger.info("Checkpoint saved: %s", path)
        self._rotate()

    def wait(self) -> None:
        if self._pending is not None:
            self._pending.join()
            self._pending = None

    def load_latest(self, model: nn.Module, optimizer: Optional[torch.optim.Optimizer] = None,
                    map_location: Optional[Any] = None) -> Optional[Dict[str, Any]]:
        files = self.list_checkpoints()
        if not files:
            return None
        return self.load(files[-1], model, optimizer, map_location)

    def load(self, path: str, model: nn.Module, optimizer: Optional[torch.optim.Optimizer] = None,
             map_location: Optional[Any] = None) -> Dict[str, Any]:
        from olympus.core.stateful_module import StatefulModule

        self.wait()
        ckpt = torch.load(path, map_location=map_location, weights_only=False)
        sd = dict(ckpt["model_state_dict"])
        has_extras = any(k.startswith("_olympus_") or k == "__stateful_states__" for k in sd)
        if isinstance(model, StatefulModule) and has_extras:
            sd.pop("__stateful_states__", None)
            model.load_state_dict_with_state(sd)
        else:
            for k in [k for k in sd if k.startswith("_olympus_") or k == "__stateful_states__"]:
                sd.pop(k)
            model.load_state_dict(sd)
        if optimizer is not None and "optimizer_state_dict" in ckpt:
            optimizer.load_state_dict(ckpt["optimizer_state_dict"])
        return ckpt

    def list_checkpoints(self) -> List[str]:
        return sorted(glob.glob(os.path.join(self.save_dir, f"{self.prefix}_step*.pt")))

    def _rotate(self) -> None:
        if self.max_to_keep <= 0:
            return
        files = self.list_checkpoints()
        for old in files[: max(0, len(files) - self.max_to_keep)]:
            try:
                os.remove(old)
            except OSError:
                pass
        self._saved = [p for p in self._saved if os.path.exists(p)]
