"""Modules that carry named state across training steps.

A :class:`StatefulModule` owns two kinds of extra tensors besides its
parameters:

* **state** -- tensors that survive from one step to the next and that can be
  pulled into the autograd graph with :meth:`StatefulModule.link_state`.  The
  gradient that reaches a linked state is accumulated on the module
  (``module._state_grads[name]``) so that an update rule can consume it.
* **memory** -- plain, non-differentiable tensors (e.g. slots shared through a
  :class:`~olympus.core.memory_bus.MemoryBus`).

Both are mirrored into registered buffers (``_state_buf_<name>`` and
``_mem_buf_<name>``) so that ``.to()``/``.cuda()`` move them and
``state_dict()`` sees them.  The checkpoint extras written by
:meth:`StatefulModule.state_dict_with_state` use the ``_olympus_*`` keys of the
reference format (``olympus/core/stateful_module.py:241-285``).
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.nn as nn

_STATE_PREFIX = "_state_buf_"
_MEMORY_PREFIX = "_mem_buf_"


class StateLink(torch.autograd.Function):
    """Identity into the graph for a persistent state tensor.

    ``forward`` returns a copy of the state (so in-place ops downstream cannot
    corrupt the stored value).  ``backward`` passes the incoming gradient
    through unchanged *and* adds it to ``module._state_grads[name]``.
    Mirrors ``olympus/core/stateful_module.py:11-55`` of the reference.
    """

    @staticmethod
    def forward(ctx, state_tensor: torch.Tensor, module_ref: Any, state_name: str) -> torch.Tensor:
        ctx.module_ref = module_ref
        ctx.state_name = state_name
        return state_tensor.clone()

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor) -> Tuple[Optional[torch.Tensor], None, None]:
        owner = ctx.module_ref
        grads = getattr(owner, "_state_grads", None)
        if grads is not None:
            prev = grads.get(ctx.state_name)
            grads[ctx.state_name] = grad_output.clone() if prev is None else prev + grad_output
        return grad_output, None, None


class StatefulModule(nn.Module):
    """``nn.Module`` with persistent, optionally gradient-linked state."""

    def __init__(self) -> None:
        super().__init__()
        self._state_tensors: Dict[str, torch.Tensor] = {}
        self._state_grads: Dict[str, Optional[torch.Tensor]] = {}
        self._memory_tensors: Dict[str, torch.Tensor] = {}
        self._state_meta: Dict[str, Dict[str, Any]] = {}
        self._memory_meta: Dict[str, Dict[str, Any]] = {}

    # ------------------------------------------------------------------ state
    def _rebind_buffer(self, buf_name: str, value: torch.Tensor, persistent: bool) -> None:
        # Re-registering (instead of copy_) lets the new value change shape,
        # which HLRT needs when the batch size of the cached plan changes.
        if buf_name in self._buffers:
            del self._buffers[buf_name]
            self._non_persistent_buffers_set.discard(buf_name)
        self.register_buffer(buf_name, value, persistent=persistent)

    def register_state(self, name: str, tensor: torch.Tensor, persistent: bool = True, **meta: Any) -> None:
        if name in self._state_tensors:
            raise ValueError(f"State '{name}' is already registered.")
        value = tensor.detach().clone()
        self._state_tensors[name] = value
        self._state_grads[name] = None
        self._state_meta[name] = {"persistent": persistent, **meta}
        self._rebind_buffer(_STATE_PREFIX + name, value, persistent)

    def _state_buffer(self, name: str) -> torch.Tensor:
        if name not in self._state_tensors:
            raise KeyError(f"State '{name}' has not been registered.")
        buf = self._buffers[_STATE_PREFIX + name]
        self._state_tensors[name] = buf
        return buf

    def link_state(self, name: str) -> torch.Tensor:
        """Return the state as a graph node whose gradient lands in ``_state_grads``."""
        return StateLink.apply(self._state_buffer(name), self, name)

    def get_state(self, name: str) -> torch.Tensor:
        return self._state_buffer(name)

    def set_state(self, name: str, value: torch.Tensor) -> None:
        if name not in self._state_tensors:
            raise KeyError(f"State '{name}' has not been registered.")
        new_val = value.detach().clone()
        self._state_tensors[name] = new_val
        self._rebind_buffer(_STATE_PREFIX + name, new_val, self._state_meta[name].get("persistent", True))

    def get_state_grad(self, name: str) -> Optional[torch.Tensor]:
        return self._state_grads.get(name)

    def zero_state_grads(self) -> None:
        for name in self._state_grads:
            self._state_grads[name] = None

    def apply_state_grads(self, lr: float = 1e-3) -> None:
        """Plain SGD step on every state that received a gradient, then clear."""
        for name, grad in list(self._state_grads.items()):
            if grad is not None:
                self.set_state(name, self.get_state(name) - lr * grad)
        self.zero_state_grads()

    # ----------------------------------------------------------------- memory
    def register_memory(self, name: str, tensor: torch.Tensor, **meta: Any) -> None:
        if name in self._memory_tensors:
            raise ValueError(f"Memory '{name}' is already registered.")
        value = tensor.detach().clone()
        self._memory_tensors[name] = value
        self._memory_meta[name] = dict(meta)
        self._rebind_buffer(_MEMORY_PREFIX + name, value, True)

    def get_memory(self, name: str) -> torch.Tensor:
        if name not in self._memory_tensors:
            raise KeyError(f"Memory '{name}' has not been registered.")
        buf = self._buffers[_MEMORY_PREFIX + name]
        self._memory_tensors[name] = buf
        return buf

    def update_memory(self, name: str, value: torch.Tensor) -> None:
        if name not in self._memory_tensors:
            raise KeyError(f"Memory '{name}' has not been registered.")
        new_val = value.detach().clone()
        self._memory_tensors[name] = new_val
        self._rebind_buffer(_MEMORY_PREFIX + name, new_val, True)

    # ------------------------------------------------------------ checkpoints
    def _sync_from_buffers(self) -> None:
        for name in self._state_tensors:
            buf = self._buffers.get(_STATE_PREFIX + name)
            if buf is not None:
                self._state_tensors[name] = buf
        for name in self._memory_tensors:
            buf = self._buffers.get(_MEMORY_PREFIX + name)
            if buf is not None:
                self._memory_tensors[name] = buf

    def olympus_extras(self) -> Dict[str, Any]:
        """The four ``_olympus_*`` entries of the reference checkpoint layout."""
        self._sync_from_buffers()
        return {
            "_olympus_state_tensors": {k: v.detach().cpu() for k, v in self._state_tensors.items()},
            "_olympus_state_meta": self._state_meta,
            "_olympus_memory_tensors": {k: v.detach().cpu() for k, v in self._memory_tensors.items()},
            "_olympus_memory_meta": self._memory_meta,
        }

    def state_dict_with_state(self, **kwargs: Any) -> Dict[str, Any]:
        out = dict(super().state_dict(**kwargs))
        out.update(self.olympus_extras())
        return out

    def restore_olympus_extras(self, extras: Dict[str, Any]) -> None:
        state_tensors = extras.get("_olympus_state_tensors", {}) or {}
        state_meta = extras.get("_olympus_state_meta", {}) or {}
        memory_tensors = extras.get("_olympus_memory_tensors", {}) or {}
        memory_meta = extras.get("_olympus_memory_meta", {}) or {}
        for name, tensor in state_tensors.items():
            if name in self._state_tensors:
                target = self._state_tensors[name]
                self.set_state(name, tensor.to(target.device))
            else:
                self.register_state(name, tensor, **state_meta.get(name, {}))
        self._state_meta.update(state_meta)
        for name, tensor in memory_tensors.items():
            if name in self._memory_tensors:
                target = self._memory_tensors[name]
                self.update_memory(name, tensor.to(target.device))
            else:
                self.register_memory(name, tensor, **memory_meta.get(name, {}))
        self._memory_meta.update(memory_meta)

    def load_state_dict_with_state(self, state_dict: Dict[str, Any], strict: bool = True) -> None:
        extras = {k: state_dict.pop(k) for k in list(state_dict.keys()) if k.startswith("_olympus_")}
        self.restore_olympus_extras(extras)
        super().load_state_dict(state_dict, strict=strict)

    # ----------------------------------------------------------------- device
    def _apply(self, fn, recurse: bool = True):  # type: ignore[override]
        # Every device/dtype move (to, cuda, half, ...) goes through _apply;
        # re-point the name -> tensor dicts at the moved buffers afterwards.
        result = super()._apply(fn, recurse)
        self._sync_from_buffers()
        return result

    # ---------------------------------------------------------------- helpers
    def state_names(self) -> List[str]:
        return list(self._state_tensors)

    def memory_names(self) -> List[str]:
        return list(self._memory_tensors)

    def extra_repr(self) -> str:
        parts = []
        if self._state_tensors:
            parts.append("states={" + ", ".join(f"{k}: {tuple(v.shape)}" for k, v in self._state_tensors.items()) + "}")
        if self._memory_tensors:
            parts.append("memories={" + ", ".join(f"{k}: {tuple(v.shape)}" for k, v in self._memory_tensors.items()) + "}")
        return ", ".join(parts)
