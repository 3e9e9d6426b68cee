"""Top-down conditioning of the token stream by Tier 2/3 (``genesis/model/conditioning.py:15-174``).

* ``apply_cached_plan``: ``h + sigmoid(alpha) * plan`` broadcast over tokens.
* ``compute_plan_vector``: mean of the Tier-2 latents over (chunks, latents),
  then ``plan_proj``.
* ``integrate_tier3``: Tier-3 output is projected (``tier3_proj``) and
  averaged over latents into one vector per packed chunk slot; the i-th
  selected slot is added (times ``sigmoid(tier3_alpha)``) to every token of
  the chunk it maps back to.  The mapping is the reference's: for sample
  ``b`` the Tier-3 mask entries ``j`` with ``mask > 0.5`` and ``j < count_b``
  (the number of chunks escalated to Tier 2) select, in order, the original
  chunks ``t2_index[b, j]``; the i-th selection receives slot ``i``.
  The reference walks this with Python loops over batch and chunks; here it
  is a prefix sum, one scatter of slot ids and one gather on the device.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops


class TopDownConditioning(nn.Module):
    def __init__(self, d_model: int, tier2_dim: int, chunk_size: int = 32) -> None:
        super().__init__()
        self.d_model = d_model
        self.tier2_dim = tier2_dim
        self.chunk_size = chunk_size
        self.plan_proj = nn.Linear(tier2_dim, d_model, bias=False)
        self.alpha = nn.Parameter(torch.zeros(1))
        self.tier3_proj = nn.Linear(tier2_dim, d_model, bias=False)
        self.tier3_alpha = nn.Parameter(torch.zeros(1))

    def apply_cached_plan(self, tier1_out: torch.Tensor, plan_vector: torch.Tensor) -> torch.Tensor:
        if plan_vector.dim() == 2:
            plan_vector = plan_vector.unsqueeze(1)
        return tier1_out + torch.sigmoid(self.alpha) * plan_vector.to(tier1_out.dtype)

    def integrate_tier3(
        self,
        tier1_out: torch.Tensor,
        tier3_out: torch.Tensor,
        tier2_mask: torch.Tensor,
        tier3_mask: torch.Tensor,
        fixed: bool = False,
    ) -> torch.Tensor:
        """``fixed`` (an extension): Tier 3 ran on the fixed-capacity buffer of all
        ``C`` chunk slots; the slot mapping is computed at that width, with no host
        read, and selects the same chunks."""
        if tier3_out is None or tier3_out.numel() == 0:
            return tier1_out
        B, S, D = tier1_out.shape
        cs = self.chunk_size
        n3 = tier3_out.shape[1]
        chunk_cond = self.tier3_proj(tier3_out).mean(dim=2)  # (B, N3, D)

        sel2 = tier2_mask if tier2_mask.dtype == torch.bool else tier2_mask > 0.5
        if fixed:  # all C slots; slots past the reference's count are never valid
            t2_idx, t2_valid, _, _ = ops.compact_chunks_fixed(sel2)
            n2 = t2_idx.shape[1]
        else:
            t2_idx, t2_valid, n2 = ops.compact_chunks(sel2)  # (B, n2)
        C = sel2.shape[1]
        sel3 = tier3_mask if tier3_mask.dtype == torch.bool else tier3_mask > 0.5
        width = min(n2, sel3.shape[1])
        m3 = sel3[:, :width] & t2_valid[:, :width]
        rank = torch.cumsum(m3.to(torch.int32), dim=1) - 1
        keep = m3 & (rank < n3)
        # src[b, c] = slot feeding chunk c (or n3 = "none").
        src = torch.full((B, C + 1), n3, dtype=torch.long, device=tier1_out.device)
        dest = torch.where(keep, t2_idx[:, :width], torch.full_like(t2_idx[:, :width], C))
        src.scatter_(1, dest, torch.where(keep, rank.to(torch.long), torch.full_like(dest, n3)))
        src = src[:, :C]
        cond = torch.cat([chunk_cond, chunk_cond.new_zeros(B, 1, D)], dim=1)
        per_chunk = cond.gather(1, src[:, :, None].expand(B, C, D))  # (B, C, D)

        pad = C * cs - S
        x = F.pad(tier1_out, (0, 0, 0, pad)) if pad > 0 else tier1_out[:, : C * cs]
        x = x.reshape(B, C, cs, D) + torch.sigmoid(self.tier3_alpha) * per_chunk[:, :, None, :]
        x = x.reshape(B, C * cs, D)
        if C * cs >= S:
            return x[:, :S]
        return torch.cat([x, tier1_out[:, C * cs:]], dim=1)

    def compute_plan_vector(self, tier2_out: torch.Tensor, n_slots: torch.Tensor | None = None) -> torch.Tensor:
        """``n_slots`` (a device scalar, an extension): average over the first
        ``n_slots`` chunk slots only (the fixed-capacity escalation path)."""
        if n_slots is None:
            return self.plan_proj(tier2_out.mean(dim=(1, 2)))
        B, N, L, D = tier2_out.shape
        m = (torch.arange(N, device=tier2_out.device) < n_slots).to(tier2_out.dtype)
        mean = (tier2_out * m[None, :, None, None]).sum(dim=(1, 2)) / (n_slots.to(tier2_out.dtype) * L)
        return self.plan_proj(mean)
