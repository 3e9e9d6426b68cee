"""Single-parameter fused Muon step (``olympus/kernels/muon_step.py:224-256``).

``muon_step(param, grad, buf, lr, momentum, weight_decay, ns_steps)`` updates
``param`` and ``buf`` in place: fused prologue (decay, momentum, Nesterov,
``||g||``), Newton-Schulz, fused norm-matched update.  No value is read back
to the host (the reference's fused path synchronises on ``.item()``).
"""

from __future__ import annotations

import torch

from llm_research_b200 import ops

NS_A, NS_B, NS_C = ops.optim.NS_A, ops.optim.NS_B, ops.optim.NS_C
HAS_TRITON = False


def _newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    return ops.newton_schulz(G, steps=steps, eps=eps)


@torch.no_grad()
def _muon_step_pt(param, grad, momentum_buffer, lr, momentum, weight_decay, ns_steps) -> None:
    if weight_decay != 0.0:
        param.mul_(1.0 - lr * weight_decay)
    momentum_buffer.mul_(momentum).add_(grad)
    u = grad + momentum * momentum_buffer
    o = _newton_schulz(u, steps=ns_steps)
    param.add_(o * (grad.norm() / (o.norm() + 1e-8)), alpha=-lr)


@torch.no_grad()
def muon_step(param: torch.Tensor, grad: torch.Tensor, momentum_buffer: torch.Tensor, lr: float = 0.02,
              momentum: float = 0.95, weight_decay: float = 0.0, ns_steps: int = 5) -> None:
    if not param.is_cuda:
        _muon_step_pt(param, grad, momentum_buffer, lr, momentum, weight_decay, ns_steps)
        return
    from olympus.optim.muon_adamw_hybrid import muon_update_group

    muon_update_group([param], [momentum_buffer], lr, momentum, weight_decay, ns_steps, grads=[grad])
