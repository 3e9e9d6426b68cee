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


# ------------------------------------------------------ chunked linear + CE
class _LinearCEFn(torch.autograd.Function):
    """``mean CE(h W^T, targets)`` without the full ``(N, V)`` logits: rows are
    processed ``chunk`` at a time (logits GEMM, the one-pass CE kernels, and the
    chunk's dh / dW GEMMs), so only one chunk's logits exist at a time.  The
    gradients are formed in the forward (the loss is linear in its upstream
    gradient) and scaled in the backward."""

    @staticmethod
    def forward(ctx, h, w, targets, ignore_index, chunk):
        N, d = h.shape
        V = w.shape[0]
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        count = (targets != ignore_index).sum().clamp_min(1).float()
        inv = (1.0 / count).reshape(1)
        loss_sum = torch.zeros((), dtype=torch.float32, device=h.device)
        dh = torch.empty_like(h) if need_h else None
        dw = torch.zeros(V, d, dtype=torch.float32, device=h.device) if need_w else None
        for s in range(0, N, chunk):
            hc, tc = h[s:s + chunk], targets[s:s + chunk].contiguous()
            logits = F.linear(hc, w)
            if logits.is_cuda:
                ls, _, lse = native().ce_fwd(logits.contiguous(), tc, int(ignore_index))
                loss_sum += ls.reshape(())
                if need_h or need_w:
                    dl = native().ce_bwd(logits.contiguous(), tc, lse, inv, int(ignore_index))
            else:
                lf = logits.float()
                valid = tc != ignore_index
                lse = torch.logsumexp(lf, dim=-1)
                tgt = lf.gather(1, tc.clamp(0, V - 1)[:, None]).squeeze(1)
                loss_sum += ((lse - tgt) * valid).sum()
                if need_h or need_w:
                    p = torch.softmax(lf, dim=-1)
                    p[torch.arange(p.shape[0]), tc.clamp(0, V - 1)] -= 1.0
                    dl = (p * (valid.float() * inv)[:, None]).to(logits.dtype)
            if need_h:
                dh[s:s + chunk] = dl @ w
            if need_w:
                dw += (dl.t() @ hc).float()
            del logits
        ctx.save_for_backward(dh, dw)
        ctx.w_dtype = w.dtype
        return loss_sum / count

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        gh = (dh * g.to(dh.dtype)) if dh is not None else None
        gw = (dw * g.float()).to(ctx.w_dtype) if dw is not None else None
        return gh, gw, None, None, None


def linear_cross_entropy(h: torch.Tensor, w: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                         chunk: int = 8192) -> torch.Tensor:
    """``cross_entropy(h @ w.T, targets)`` (mean over targets != ignore_index) with the
    logits formed ``chunk`` rows at a time.  ``h (N, d)``, ``w (V, d)``, ``targets (N,)``."""
    return _LinearCEFn.apply(h.reshape(-1, h.shape[-1]), w, targets.reshape(-1), ignore_index, int(chunk))
