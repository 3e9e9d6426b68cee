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

:func:`vocab_parallel_linear_cross_entropy` is the head + loss for tensor
parallelism: every rank of the group multiplies the (replicated) hidden states
by its ``V / tp`` rows of the head weight only, the per-row log-sum-exp and
target logit are combined over the group, and the gradients come back
replicated (``dh`` summed over the shards, ``dW`` gathered from them).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

import torch.distributed as dist

from llm_research_b200._ext import native
from llm_research_b200.ops.linear import _pair_ok, _rows


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
        pair = h.is_cuda and _pair_ok(h, w)
        if pair:
            from llm_research_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad
        for s in range(0, N, chunk):
            hc, tc = h[s:s + chunk], targets[s:s + chunk].contiguous()
            logits = linear_fwd(_rows(hc), w) if pair else F.linear(hc, w)
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
                if pair:
                    linear_dgrad(dl, w, out=dh[s:s + chunk])
                else:
                    dh[s:s + chunk] = dl @ w
            if need_w:
                if pair:  # fp32 accumulation in the GEMM epilogue
                    linear_wgrad(dl, _rows(hc), out=dw, accumulate=True)
                else:
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


# ------------------------------------------------ vocabulary-parallel linear + CE
def vocab_shard_range(V: int, world: int, rank: int):
    """Rows ``[v0, v1)`` of the head owned by ``rank``: ``ceil(V / world)`` per rank,
    the last shard shorter when it does not divide."""
    per = (V + world - 1) // world
    v0 = min(rank * per, V)
    return v0, min(v0 + per, V), per


class _VocabParallelLinearCEFn(torch.autograd.Function):
    """Each rank forms ``h W_r^T`` for its vocabulary rows ``W_r``, one chunk of
    rows at a time, and keeps those local logits.  One all-gather of the per-row
    ``(local lse, local target logit)`` pairs gives the full-vocabulary
    log-sum-exp and the target logit, hence the loss (identical on every rank).
    The local logits' gradient ``softmax - onehot`` (one-hot only on the owning
    shard) gives this rank's share of ``dh`` and its rows of ``dW``; backward sums
    ``dh`` and all-gathers ``dW`` over the group."""

    @staticmethod
    def forward(ctx, h, w, targets, ignore_index, chunk, group):
        N, d = h.shape
        V = w.shape[0]
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        v0, v1, per = vocab_shard_range(V, world, rank)
        w_loc = w[v0:v1]
        valid = targets != ignore_index
        owned = valid & (targets >= v0) & (targets < v1)
        # Rows whose target lives on another shard get a sentinel outside
        # [0, v1 - v0) that also differs from ignore_index, so the shard kernels
        # count them (softmax gradient, no one-hot) instead of ignoring them.
        other = -2 if ignore_index == -1 else -1
        t_loc = torch.where(owned, targets - v0, torch.where(valid, torch.full_like(targets, other), targets))
        stats = torch.zeros(2, N, dtype=torch.float32, device=h.device)  # (local lse, local target logit)
        logits = []
        empty = v1 == v0  # V < world * ceil(V / world): the last ranks own no rows
        if empty:
            stats[0].fill_(float("-inf"))  # log-sum-exp over an empty set of logits
        pair = h.is_cuda and not empty and _pair_ok(h, w_loc)
        if pair:
            from llm_research_b200.ops.gemm import linear_dgrad, linear_fwd, linear_wgrad
        for s in range(0, 0 if empty else N, chunk):
            lg = linear_fwd(_rows(h[s:s + chunk]), w_loc) if pair else F.linear(h[s:s + chunk], w_loc).contiguous()
            tc = t_loc[s:s + chunk].contiguous()
            if lg.is_cuda:
                _, _, lse = native().ce_fwd(lg, tc, int(ignore_index))
                stats[0, s:s + chunk] = lse
            else:
                stats[0, s:s + chunk] = torch.logsumexp(lg.float(), dim=-1)
            tl = lg.gather(1, tc.clamp(0, max(v1 - v0 - 1, 0))[:, None]).squeeze(1).float()
            stats[1, s:s + chunk] = torch.where(owned[s:s + chunk], tl, torch.zeros_like(tl))
            logits.append(lg)
        gathered = torch.empty(world * 2, N, dtype=torch.float32, device=h.device)
        dist.all_gather_into_tensor(gathered, stats, group=group)
        gathered = gathered.view(world, 2, N)
        lse = torch.logsumexp(gathered[:, 0], dim=0)
        tgt = gathered[:, 1].sum(0)
        count = valid.sum().clamp_min(1).float()
        loss = ((lse - tgt) * valid).sum() / count
        inv = (1.0 / count).reshape(1)
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dh = torch.zeros_like(h) if need_h else None
        dw = torch.zeros(per, d, dtype=torch.float32, device=h.device) if need_w else None
        for i, s in enumerate(range(0, 0 if empty else N, chunk)):
            lg, tc = logits[i], t_loc[s:s + chunk].contiguous()
            if not (need_h or need_w):
                break
            if lg.is_cuda:
                dl = native().ce_bwd_vocab_shard(lg, tc, lse[s:s + chunk].contiguous(), inv, int(ignore_index))
            else:
                p = torch.exp(lg.float() - lse[s:s + chunk, None])
                own = owned[s:s + chunk]
                rows = torch.arange(p.shape[0], device=p.device)[own]
                p[rows, tc[own]] -= 1.0
                dl = (p * (valid[s:s + chunk].float() * inv)[:, None]).to(lg.dtype)
            if need_h:
                if pair:
                    linear_dgrad(dl, w_loc, out=dh[s:s + chunk])
                else:
                    dh[s:s + chunk] = dl @ w_loc
            if need_w:
                if pair:
                    linear_wgrad(dl, _rows(h[s:s + chunk]), out=dw[: v1 - v0], accumulate=True)
                else:
                    dw[: v1 - v0] += (dl.t() @ h[s:s + chunk]).float()
            logits[i] = None
        ctx.save_for_backward(dh, dw)
        ctx.group, ctx.V, ctx.w_dtype = group, V, w.dtype
        return loss

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        gh = gw = None
        if dh is not None:
            gh = dh * g.to(dh.dtype)
            dist.all_reduce(gh, group=ctx.group)
        if dw is not None:
            world = dist.get_world_size(ctx.group)
            part = (dw * g.float()).to(ctx.w_dtype)
            full = torch.empty(world * part.shape[0], part.shape[1], dtype=ctx.w_dtype, device=part.device)
            dist.all_gather_into_tensor(full, part, group=ctx.group)
            gw = full[: ctx.V]
        return gh, gw, None, None, None, None


def vocab_parallel_linear_cross_entropy(h: torch.Tensor, w: torch.Tensor, targets: torch.Tensor,
                                        group: dist.ProcessGroup, ignore_index: int = -100,
                                        chunk: int = 8192) -> torch.Tensor:
    """``cross_entropy(h @ w.T, targets)`` over a tensor-parallel group: ``h (N, d)``,
    ``w (V, d)`` and ``targets (N,)`` are replicated on the group's ranks, each rank
    multiplies by ``V / tp`` rows of ``w``; the loss and both gradients come back
    replicated."""
    return _VocabParallelLinearCEFn.apply(h.reshape(-1, h.shape[-1]), w, targets.reshape(-1), ignore_index,
                                          int(chunk), group)
