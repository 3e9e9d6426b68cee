"""Run the reference implementation in a separate interpreter as a numerical oracle.

The reference's packages share their top-level names (``genesis``,
``olympus``) with this repository, so they are imported in a child process
whose ``sys.path`` holds only the reference installation.  Results come back
through a ``torch.save`` file.
"""

from __future__ import annotations

import os
import subprocess
import sys
import tempfile
from typing import Any, Dict, Optional

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
# The installed reference (``baseline/_ref``, made by ``__graft_entry__.build``)
# or a source tree named by ``LRB_REFERENCE_DIR``.
CANDIDATES = [p for p in (os.environ.get("LRB_REFERENCE_DIR"), os.path.join(REPO, "baseline", "_ref")) if p]


def reference_root() -> Optional[str]:
    for c in CANDIDATES:
        if os.path.isdir(os.path.join(c, "genesis")) and os.path.isdir(os.path.join(c, "olympus")):
            return c
    return None


_CHILD = r"""
import sys, torch
root, job, out = sys.argv[1], sys.argv[2], sys.argv[3]
sys.path[:] = [root] + [p for p in sys.path if 'repo' not in p]
spec = torch.load(job, weights_only=False)
ns = {}
exec(spec['code'], ns)
res = ns['run'](spec.get('args', {}))
torch.save(res, out)
"""


def run_reference(code: str, args: Dict[str, Any] | None = None, timeout: float = 600.0) -> Any:
    """Execute ``code`` (which must define ``run(args) -> result``) against the reference."""
    root = reference_root()
    if root is None:
        raise FileNotFoundError("reference implementation not found")
    with tempfile.TemporaryDirectory() as d:
        job, out = os.path.join(d, "job.pt"), os.path.join(d, "out.pt")
        torch.save({"code": code, "args": args or {}}, job)
        env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=root)
        proc = subprocess.run([sys.executable, "-c", _CHILD, root, job, out], capture_output=True, text=True,
                              timeout=timeout, env=env, cwd=d)
        if proc.returncode != 0:
            raise RuntimeError(f"reference run failed:\n{proc.stderr[-3000:]}")
        return torch.load(out, weights_only=False)
