"""Verifier → generator distillation (``genesis/verifier/distillation.py:16-133``).

``distillation_loss``: MSE between ``proj_G(h_G)`` and ``proj_V(h_V)`` in a
shared space, the verifier side detached.  ``temperature_scaled_loss``:
``T² · KL(softmax(v/T) ‖ softmax(g/T))`` with batch-mean reduction.
``forward`` returns the MSE term (the KL term is called explicitly when
logits exist).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class VerificationDistillation(nn.Module):
    def __init__(self, generator_dim: int, verifier_dim: int, shared_dim: int = 256, alpha: float = 0.5) -> None:
        super().__init__()
        self.generator_dim = generator_dim
        self.verifier_dim = verifier_dim
        self.shared_dim = shared_dim
        self.alpha = alpha
        self.proj_G = nn.Linear(generator_dim, shared_dim)
        self.proj_V = nn.Linear(verifier_dim, shared_dim)
        for lin in (self.proj_G, self.proj_V):
            nn.init.xavier_uniform_(lin.weight)
            nn.init.zeros_(lin.bias)

    def distillation_loss(self, generator_hidden: torch.Tensor, verifier_hidden: torch.Tensor) -> torch.Tensor:
        return F.mse_loss(self.proj_G(generator_hidden), self.proj_V(verifier_hidden).detach())

    def temperature_scaled_loss(self, g_logits: torch.Tensor, v_logits: torch.Tensor,
                                temperature: float = 2.0) -> torch.Tensor:
        g = F.log_softmax(g_logits.float() / temperature, dim=-1)
        v = F.softmax(v_logits.float() / temperature, dim=-1).detach()
        return F.kl_div(g, v, reduction="batchmean") * (temperature ** 2)

    def forward(self, generator_hidden: torch.Tensor, verifier_hidden: torch.Tensor) -> torch.Tensor:
        return self.distillation_loss(generator_hidden, verifier_hidden)
