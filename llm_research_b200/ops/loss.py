"""Token cross-entropy, one pass each way, without copying the logits.

``loss = mean over rows with target != ignore_index of (lse(row) - row[target])``
in fp32 from bf16/fp32 logits (``F.cross_entropy`` semantics used by
``genesis/training/train_phase1_bootstrap.py:74-78``).  The forward keeps only
the per-row log-sum-exp; the backward writes ``(softmax - onehot) * g / n``
in the logits dtype.

:func:`shifted_cross_entropy` is the next-token loss on the *unshifted*
``(B, S, V)`` logits: row ``(b, t)`` is scored against ``ids[b, t+1]`` and the
last position of every sequence is ignored.  This equals the reference's
``cross_entropy(logits[:, :-1].contiguous(), ids[:, 1:])`` without the copy of
the shifted logits (and its zero-padded gradient).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from llm_research_b200._ext import native


class _CEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index):
        loss_sum, count, lse = native().ce_fwd(logits, targets, int(ignore_index))
        ctx.save_for_backward(logits, targets, lse, count)
        ctx.ignore_index = ignore_index
        return loss_sum / count.clamp_min(1)

    @staticmethod
    def backward(ctx, g):
        logits, targets, lse, count = ctx.saved_tensors
        scale = g.float() / count.clamp_min(1)
        dlogits = native().ce_bwd(logits, targets, lse, scale, int(ctx.ignore_index))
        return dlogits, None, None


def cross_entropy(logits: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    V = logits.shape[-1]
    if not logits.is_cuda:
        return F.cross_entropy(logits.reshape(-1, V).float(), targets.reshape(-1), ignore_index=ignore_index)
    return _CEFn.apply(logits.reshape(-1, V).contiguous(), targets.reshape(-1).contiguous(), ignore_index)


def shifted_cross_entropy(logits: torch.Tensor, input_ids: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
    B, S, V = logits.shape
    if not logits.is_cuda:
        return F.cross_entropy(
            logits[:, :-1].reshape(-1, V).float(), input_ids[:, 1:].reshape(-1), ignore_index=ignore_index
        )
    targets = torch.cat([input_ids[:, 1:], input_ids.new_full((B, 1), ignore_index)], dim=1)
    return _CEFn.apply(logits.reshape(B * S, V).contiguous(), targets.reshape(-1).contiguous(), ignore_index)
