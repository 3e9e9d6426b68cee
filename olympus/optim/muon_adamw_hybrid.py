"""Muon for well-shaped matrices, AdamW for everything else.

Routing (``olympus/optim/muon_adamw_hybrid.py:109-116``): a parameter goes to
Muon iff it is 2-D and ``max(shape) <= min(shape) * muon_max_aspect_ratio``;
all others (biases, norms, very wide embeddings) use bias-corrected AdamW with
decoupled weight decay.  Group keys and per-parameter state keys
(``{"type": "muon", "momentum_buffer"}`` / ``{"type": "adamw", "step",
"exp_avg", "exp_avg_sq"}``) follow the reference checkpoint layout.

Execution is batched instead of one parameter at a time: every Muon matrix of
a group runs through one fused prologue (weight decay, momentum, Nesterov,
gradient norm), the Newton-Schulz iterations run batched over all matrices of
the same shape, and one fused epilogue applies the norm-matched update.  All
AdamW parameters of a group are updated by one multi-tensor kernel.  Nothing
reads a value back to the host.
"""

from __future__ import annotations

from collections import defaultdict
from typing import Dict, List, Sequence, Tuple

import torch
from torch.optim import Optimizer

from llm_research_b200 import ops


def uses_muon(p: torch.Tensor, max_aspect_ratio: float) -> bool:
    return p.dim() == 2 and max(p.shape) <= min(p.shape) * max_aspect_ratio


@torch.no_grad()
def muon_update_group(
    params: Sequence[torch.Tensor],
    bufs: Sequence[torch.Tensor],
    lr: float,
    momentum: float,
    weight_decay: float,
    ns_steps: int,
    grads: Sequence[torch.Tensor] | None = None,
) -> None:
    """Apply one Muon step to every ``params[i]`` (2-D) with momentum ``bufs[i]``."""
    if not params:
        return
    grads = [p.grad for p in params] if grads is None else list(grads)
    # 1+2: decay, momentum, Nesterov direction and ||g|| (fused per tensor).
    nesterov, gnorms = ops.muon_prologue(list(params), grads, list(bufs), lr, momentum, weight_decay)
    # 3: batched Newton-Schulz over equal shapes.
    by_shape: Dict[Tuple[int, int], List[int]] = defaultdict(list)
    for i, u in enumerate(nesterov):
        by_shape[tuple(u.shape)].append(i)
    orth: List[torch.Tensor] = [None] * len(params)  # type: ignore[list-item]
    for shape, idx in by_shape.items():
        stacked = torch.stack([nesterov[i] for i in idx]) if len(idx) > 1 else nesterov[idx[0]].unsqueeze(0)
        out = ops.newton_schulz(stacked, steps=ns_steps)
        for j, i in enumerate(idx):
            orth[i] = out[j]
    # 4+5: p -= lr * ||g|| / (||o|| + 1e-8) * o
    ops.muon_epilogue(list(params), orth, gnorms, lr)


class MuonAdamWHybrid(Optimizer):
    def __init__(
        self,
        params,
        lr_muon: float = 0.02,
        lr_adamw: float = 3e-4,
        momentum: float = 0.95,
        betas: tuple = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay_muon: float = 0.0,
        weight_decay_adamw: float = 0.01,
        ns_steps: int = 5,
        muon_max_aspect_ratio: float = 8.0,
    ) -> None:
        defaults = dict(
            lr_muon=lr_muon,
            lr_adamw=lr_adamw,
            momentum=momentum,
            betas=betas,
            eps=eps,
            weight_decay_muon=weight_decay_muon,
            weight_decay_adamw=weight_decay_adamw,
            ns_steps=ns_steps,
            muon_max_aspect_ratio=muon_max_aspect_ratio,
        )
        super().__init__(params, defaults)

    @staticmethod
    def _newton_schulz(G: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
        return ops.newton_schulz(G, steps=steps, eps=eps)

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            muon_p, muon_buf = [], []
            adam_p, adam_g, adam_m, adam_v, adam_steps = [], [], [], [], []
            for p in group["params"]:
                if p.grad is None:
                    continue
                st = self.state[p]
                if uses_muon(p, group["muon_max_aspect_ratio"]):
                    if len(st) == 0:
                        st["type"] = "muon"
                        st["momentum_buffer"] = torch.zeros_like(p.grad)
                    muon_p.append(p)
                    muon_buf.append(st["momentum_buffer"])
                else:
                    if len(st) == 0:
                        st["type"] = "adamw"
                        st["step"] = 0
                        st["exp_avg"] = torch.zeros_like(p)
                        st["exp_avg_sq"] = torch.zeros_like(p)
                    st["step"] += 1
                    adam_p.append(p)
                    adam_g.append(p.grad)
                    adam_m.append(st["exp_avg"])
                    adam_v.append(st["exp_avg_sq"])
                    adam_steps.append(st["step"])
            muon_update_group(
                muon_p, muon_buf, group["lr_muon"], group["momentum"], group["weight_decay_muon"], group["ns_steps"]
            )
            if adam_p:
                beta1, beta2 = group["betas"]
                ops.adamw_step(
                    adam_p, adam_g, adam_m, adam_v, adam_steps,
                    lr=group["lr_adamw"], beta1=beta1, beta2=beta2, eps=group["eps"],
                    weight_decay=group["weight_decay_adamw"],
                )
        return loss
