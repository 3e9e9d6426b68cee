"""Muon: momentum orthogonalised by a Newton-Schulz iteration.

Update rule (``olympus/optim/muon.py:106-157`` of the reference), per 2-D
parameter ``p`` with gradient ``g``:

1. decoupled weight decay ``p *= 1 - lr * wd``;
2. ``buf = mu * buf + g`` and the Nesterov look-ahead ``u = g + mu * buf``;
3. ``o = NS5(u)`` -- five steps of the quintic iteration
   ``X <- a X + b (X X^T) X + c (X X^T)^2 X`` with
   ``(a, b, c) = (3.4445, -4.7750, 2.0315)`` after Frobenius normalisation;
4. rescale ``o *= ||g|| / (||o|| + 1e-8)``;
5. ``p -= lr * o``.

Orientation: the polynomial is applied through the Gram matrix of the *short*
side.  For a tall ``X`` (m > n) the reference forms the m x m matrix
``X X^T``; ``(X X^T)^k X = X (X^T X)^k`` so using the n x n Gram gives the same
polar-factor iterate with ``(n/m)`` of the FLOPs.  On CUDA the iteration runs
in bf16 on the tensor cores (the sm_100a batched Newton-Schulz in
``llm_research_b200.ops.newton_schulz``); on CPU it runs in fp32.
"""

from __future__ import annotations

from typing import Iterable, List

import torch
from torch.optim import Optimizer

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7, dtype: torch.dtype | None = None) -> torch.Tensor:
    """Orthogonalise ``G`` (2-D, or a batch ``(..., m, n)``); returns ``G``'s shape/dtype."""
    from llm_research_b200.ops import newton_schulz as ns_op

    return ns_op(G, steps=steps, eps=eps, compute_dtype=dtype)


class Muon(Optimizer):
    def __init__(self, params: Iterable, lr: float = 0.02, momentum: float = 0.95, weight_decay: float = 0.0, ns_steps: int = 5) -> None:
        if lr < 0.0:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= momentum < 1.0:
            raise ValueError(f"Invalid momentum: {momentum}")
        super().__init__(params, dict(lr=lr, momentum=momentum, weight_decay=weight_decay, ns_steps=ns_steps))
        for group in self.param_groups:
            for p in group["params"]:
                if p.dim() != 2:
                    raise ValueError(
                        f"Muon only supports 2-D parameters, got shape {tuple(p.shape)}. "
                        "Use MuonAdamWHybrid for mixed-dimension parameter sets."
                    )

    @staticmethod
    def _newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
        return newton_schulz(G, steps=steps, eps=eps)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        from olympus.optim.muon_adamw_hybrid import muon_update_group

        for group in self.param_groups:
            params: List[torch.Tensor] = [p for p in group["params"] if p.grad is not None]
            bufs = []
            for p in params:
                st = self.state[p]
                if len(st) == 0:
                    st["momentum_buffer"] = torch.zeros_like(p.grad)
                bufs.append(st["momentum_buffer"])
            muon_update_group(params, bufs, group["lr"], group["momentum"], group["weight_decay"], group["ns_steps"])
        return loss
