"""Loader for the sm_100a extension ``llm_research_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace``) so the
shared object travels with the source tree.  CUDA tensors are only ever
handled by the native kernels: if the extension cannot be imported while a
CUDA tensor reaches an op, :func:`native` raises instead of silently running a
PyTorch fallback.  CPU tensors use the PyTorch reference path of each op.
"""

from __future__ import annotations

import importlib
import os
from typing import Any, Optional

_mod: Optional[Any] = None
_err: Optional[BaseException] = None


def _load() -> Optional[Any]:
    global _mod, _err
    if _mod is not None or _err is not None:
        return _mod
    try:
        import torch  # noqa: F401  (loads libtorch before the extension)

        _mod = importlib.import_module("llm_research_b200._C")
    except BaseException as exc:  # ImportError, OSError (missing symbols), ...
        _err = exc
    return _mod


def available() -> bool:
    return _load() is not None


def native() -> Any:
    """Return the extension module or raise a descriptive error."""
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "llm_research_b200._C (the sm_100a kernels) is not built or failed to load: "
            f"{_err!r}. Build it with `python setup.py build_ext --inplace` in {os.path.dirname(os.path.dirname(__file__))}."
        )
    return mod


def load_error() -> Optional[BaseException]:
    _load()
    return _err
