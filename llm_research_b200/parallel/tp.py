"""Tensor parallelism (Megatron column / row split) with sequence parallelism,
on the fused GEMM + collective kernels of ``csrc/comm/gemm_comm.cu``.

Activations between layers are sharded along tokens (sequence parallel):
``x_shard`` is ``(T / tp, d)`` on every rank.

* :class:`ColumnParallelLinear` (QKV, up/gate): ``y = AllGather_T(x) W_r^T``
  with ``W_r`` the rank's ``out / tp`` rows.  Forward = ``ag_gemm`` (copy CTAs
  pull peer chunks into a local buffer while the tensor-core CTAs consume
  them); backward dX = ``gemm_rs`` (dY W_r, reduce-scattered over tokens by
  the epilogue's stores into the owners' slots), dW = dYᵀ AllGather(x).
* :class:`RowParallelLinear` (o_proj, down): ``y_shard = ReduceScatter_T(x W_r^T)``
  with ``W_r`` the rank's ``in / tp`` columns.  Forward = ``gemm_rs`` +
  ``tp_reduce`` (fp32 sum of the slots, optional fused residual add);
  backward dX = ``ag_gemm`` (AllGather(dY) W_r), dW = AllGather(dY)ᵀ x.

Buffers live in one :class:`~llm_research_b200.parallel.symm.SymmetricHeap`
per TP group (:class:`TPComm`).  Every call bumps an epoch that all ranks
share (calls are collective and in the same order); ``gemm_rs`` slots are
released by the owner's ``consumed`` flag, ``ag_gemm`` source shards are
double-buffered by epoch parity: a rank republishes slot ``e % 2`` only after
its own ``ag_gemm(e-1)``, which waited for every peer's ``e-1`` publish, which
each peer issued after finishing its ``ag_gemm(e-2)`` reads of that slot
(one stream per rank).

Backward GEMMs: the weight gradients run on the CTA-pair kernel from the rows
the fused forward gathered anyway (``ag_gemm`` keeps its gathered input), with
direct fp32 accumulation into the sharding engine's gradient buffer, so no
collective and no library GEMM runs for them.

Under NVFP4 linear precision (or shapes the fused kernels do not take) a layer
is ``project`` -- NVFP4 forward, dgrad and wgrad on the block-scaled kernel --
composed with differentiable row all-gather / reduce-scatter functions that
use this heap's P2P kernels (``shard_publish`` + ``p2p_pull``;
``p2p_rows_rs_push`` + ``p2p_rows_rs_reduce`` with the residual added in the
reduction).

Without a heap (CPU, several nodes, or ``comm="nccl"``) the same composition
runs NCCL / gloo collectives -- the baseline.
"""

from __future__ import annotations

import contextlib
import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200._ext import native
from llm_research_b200.ops.linear import project
from llm_research_b200.utils.nvtx import nvtx_fn


class TPComm:
    """Symmetric buffers for TP collectives of up to ``max_tokens`` tokens and ``max_width`` features."""

    def __init__(self, group: Optional[dist.ProcessGroup], max_tokens: int, max_width: int,
                 device: torch.device, ncopy: int = 16) -> None:
        from llm_research_b200.parallel.symm import SymmetricHeap

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device
        self.max_tokens, self.max_width, self.ncopy = max_tokens, max_width, ncopy
        W = self.world
        # gemm_rs slots are tile-major with the width padded to whole 256-column tiles
        slot = (max_tokens // W) * (-(-max_width // 256) * 256) * 2
        self.heap = h = SymmetricHeap(3 * W * slot + 2 * slot + 16384, group=group, device=device)
        # gemm_rs receive slots, two sets alternating by epoch parity (a call only waits
        # for the owners to have consumed the call before the previous one)
        self.recv_offs = [h.alloc(W * slot), h.alloc(W * slot)]
        self.ready_off = h.alloc(4 * W)
        self.consumed_off = h.alloc(4)
        self.shard_off = [h.alloc(slot), h.alloc(slot)]
        self.shard_ready_off = [h.alloc(4), h.alloc(4)]
        self.ready = h.view(self.ready_off, (W,), torch.int32)
        self.consumed = h.view(self.consumed_off, (1,), torch.int32)
        self.shard_ready = [h.view(o, (1,), torch.int32) for o in self.shard_ready_off]
        self.counters = torch.zeros(W + 4, dtype=torch.int32, device=device)
        self.chunk_flags = torch.zeros(max_tokens // 128, dtype=torch.int32, device=device)
        self.rs_epoch = 0
        self.ag_epoch = 0
        # row reduce-scatter outside the fused GEMMs: one receive region, released
        # by each owner's consumed flag before the next push
        self.rrs_recv_off = h.alloc(W * slot)
        self.rrs_ready_off = h.alloc(4 * W)
        self.rrs_consumed_off = h.alloc(4)
        self.rrs_recv = h.view(self.rrs_recv_off, (W * slot // 2,), torch.bfloat16)
        self.rrs_ready = h.view(self.rrs_ready_off, (W,), torch.int32)
        self.rrs_consumed = h.view(self.rrs_consumed_off, (1,), torch.int32)
        self.rrs_counters = torch.zeros(2, dtype=torch.int32, device=device)
        self.rrs_epoch = 0
        self._slot_bytes = slot

    @nvtx_fn("lrb/tp/gemm_rs")
    def gemm_rs(self, x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``ReduceScatter_rows(x @ w.T)`` (+ residual): ``(T, K) x (N, K) -> (T / world, N)``."""
        C = native()
        T, N = x.shape[0], w.shape[0]
        self.rs_epoch += 1
        recv_off = self.recv_offs[self.rs_epoch % 2]
        C.gemm_rs(x.contiguous(), w, self.heap.bases, recv_off, self.ready_off, self.consumed_off, self.rank,
                  self.world, self.rs_epoch, self.counters[: self.world], self.heap.err)
        out = torch.empty(T // self.world, N, dtype=x.dtype, device=x.device)
        npad = -(-N // 256) * 256
        recv = self.heap.view(recv_off, (self.world * (T // self.world) * npad,), torch.bfloat16)
        C.tp_reduce(recv, residual.contiguous() if residual is not None else None, out, self.world, self.ready,
                    self.consumed, self.rs_epoch, self.counters[self.world:self.world + 1], self.heap.err)
        return out

    def _publish(self, x_shard: torch.Tensor) -> int:
        """Copy this rank's rows into the shard slot of the next gather epoch."""
        Tl, K = x_shard.shape
        self.ag_epoch += 1
        s = self.ag_epoch % 2
        dst = self.heap.view(self.shard_off[s], (Tl, K), x_shard.dtype)
        native().shard_publish(x_shard.contiguous(), dst, self.shard_ready[s], self.ag_epoch,
                               self.counters[self.world + 1:self.world + 2])
        return s

    @nvtx_fn("lrb/tp/ag_gemm")
    def ag_gemm(self, x_shard: torch.Tensor, w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """``AllGather_rows(x_shard) @ w.T``: ``(T / world, K) x (N, K) -> (T, N)``,
        and the gathered ``(T, K)`` rows (the weight gradient's operand)."""
        Tl, K = x_shard.shape
        s = self._publish(x_shard)
        a_full = torch.empty(Tl * self.world, K, dtype=x_shard.dtype, device=x_shard.device)
        y = native().ag_gemm(w, a_full, self.chunk_flags, self.heap.bases, self.shard_off[s], self.shard_ready_off[s],
                             self.rank, self.world, self.ag_epoch, self.ncopy, self.heap.err)
        return y, a_full

    @nvtx_fn("lrb/tp/all_gather")
    def all_gather(self, x_shard: torch.Tensor) -> torch.Tensor:
        """Rows of every rank, P2P pulls from the peers' shard slots."""
        Tl, K = x_shard.shape
        s = self._publish(x_shard)
        out = torch.empty(Tl * self.world, K, dtype=x_shard.dtype, device=x_shard.device)
        native().p2p_pull(out, self.heap.bases, self.shard_off[s], self.shard_ready_off[s], self.world,
                          self.ag_epoch, self.heap.err)
        return out

    @nvtx_fn("lrb/tp/reduce_scatter")
    def reduce_scatter(self, y: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """This rank's rows of the sum over ranks of ``y`` (+ ``residual``)."""
        C = native()
        T, N = y.shape
        self.rrs_epoch += 1
        C.p2p_rows_rs_push(y.contiguous(), self.heap.bases, self.rrs_recv_off, self.rrs_ready_off,
                           self.rrs_consumed_off, self.rank, self.world, self.rrs_epoch, self.rrs_counters[0:1],
                           self.heap.err)
        out = torch.empty(T // self.world, N, dtype=y.dtype, device=y.device)
        C.p2p_rows_rs_reduce(self.rrs_recv, residual.contiguous() if residual is not None else None, out, self.world,
                             self.rrs_ready, self.rrs_consumed, self.rrs_epoch, self.rrs_counters[1:2], self.heap.err)
        return out

    def fits(self, tokens: int, width: int) -> bool:
        return (tokens <= self.max_tokens and width <= self.max_width and tokens % (128 * self.world) == 0
                and width % 8 == 0)

    def fits_rows(self, t: torch.Tensor, tokens: int) -> bool:
        """``t`` (rows of a ``tokens``-row matrix) can use the P2P gather / reduce-scatter."""
        return (t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 2 and tokens <= self.max_tokens
                and t.shape[1] <= self.max_width and (tokens * t.shape[1]) % (8 * self.world) == 0)

    def close(self) -> None:
        self.heap.close()


# ----------------------------------------------------------- collectives (fallback)
def _all_gather_rows(x: torch.Tensor, group) -> torch.Tensor:
    W = dist.get_world_size(group)
    out = torch.empty(x.shape[0] * W, *x.shape[1:], dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _reduce_scatter_rows(x: torch.Tensor, group) -> torch.Tensor:
    W = dist.get_world_size(group)
    out = torch.empty(x.shape[0] // W, *x.shape[1:], dtype=x.dtype, device=x.device)
    if x.is_cuda:
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    else:  # gloo has no reduce_scatter_tensor
        full = x.contiguous().clone()
        dist.all_reduce(full, group=group)
        out.copy_(full.chunk(W)[dist.get_rank(group)])
    return out


def _fused_ok(comm: Optional[TPComm], x: torch.Tensor, tokens: int, widths) -> bool:
    # The fused kernels multiply in bf16; under NVFP4 linear precision the layers
    # take the collective path around the NVFP4 GEMM instead.
    from llm_research_b200.ops.linear import get_linear_precision

    return (comm is not None and x.is_cuda and x.dtype == torch.bfloat16 and get_linear_precision() == "bf16"
            and all(comm.fits(tokens, w) for w in widths))


def _gather_rows(x_shard: torch.Tensor, comm: Optional[TPComm], group) -> torch.Tensor:
    W = dist.get_world_size(group)
    if comm is not None and comm.fits_rows(x_shard, x_shard.shape[0] * W):
        return comm.all_gather(x_shard)
    return _all_gather_rows(x_shard, group)


def _scatter_rows(y: torch.Tensor, comm: Optional[TPComm], group,
                  residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    if comm is not None and comm.fits_rows(y, y.shape[0]):
        return comm.reduce_scatter(y, residual)
    out = _reduce_scatter_rows(y, group)
    return out + residual if residual is not None else out


class _AllGatherRows(torch.autograd.Function):
    """Sequence shards -> all rows; backward reduce-scatters the gradient."""

    @staticmethod
    def forward(ctx, x_shard, comm, group):
        ctx.comm, ctx.group = comm, group
        return _gather_rows(x_shard, comm, group)

    @staticmethod
    def backward(ctx, g):
        return _scatter_rows(g.contiguous(), ctx.comm, ctx.group), None, None


class _ReduceScatterRows(torch.autograd.Function):
    """Partial products -> this rank's rows of their sum (+ residual); backward
    all-gathers the gradient (the residual's gradient passes through)."""

    @staticmethod
    def forward(ctx, y, residual, comm, group):
        ctx.comm, ctx.group, ctx.has_residual = comm, group, residual is not None
        return _scatter_rows(y, comm, group, residual)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        return _gather_rows(g, ctx.comm, ctx.group), (g if ctx.has_residual else None), None, None


def _wgrad(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``dy^T x`` on the pair kernel, added into the engine's fp32 accumulator when
    the weight carries one (the returned marker tells the engine it is done)."""
    from llm_research_b200.ops.gemm import linear_wgrad
    from llm_research_b200.ops.linear import _acc_of, accumulated_marker

    acc = _acc_of(w)
    if acc is not None:
        linear_wgrad(dy, x, out=acc, accumulate=True)
        return accumulated_marker(w)
    return linear_wgrad(dy, x).to(w.dtype)


class _ColumnFn(torch.autograd.Function):
    """Fused column-parallel layer: forward ``ag_gemm``; backward dX by ``gemm_rs``
    and dW from the rows the forward gathered."""

    @staticmethod
    def forward(ctx, x_shard, w, comm, group):
        ctx.comm, ctx.group = comm, group
        y, a_full = comm.ag_gemm(x_shard, w)
        ctx.save_for_backward(a_full, w)
        return y

    @staticmethod
    def backward(ctx, dy):
        from llm_research_b200.ops.gemm import linear_dgrad

        a_full, w = ctx.saved_tensors
        comm, group = ctx.comm, ctx.group
        dy = dy.contiguous()
        dx = None
        if ctx.needs_input_grad[0]:
            if _fused_ok(comm, dy, dy.shape[0], (w.shape[1], w.shape[0])):
                dx = comm.gemm_rs(dy, w.t().contiguous())
            else:
                dx = _scatter_rows(linear_dgrad(dy, w), comm, group)
        dw = _wgrad(dy, a_full, w) if ctx.needs_input_grad[1] else None
        return dx, dw, None, None


class _RowFn(torch.autograd.Function):
    """Fused row-parallel layer: forward ``gemm_rs`` (+ residual in the reduction);
    backward dX by ``ag_gemm`` and dW from the gradient rows it gathered."""

    @staticmethod
    def forward(ctx, x, w, residual, comm, group):
        ctx.comm, ctx.group = comm, group
        ctx.save_for_backward(x, w)
        ctx.has_residual = residual is not None
        return comm.gemm_rs(x, w, residual)

    @staticmethod
    def backward(ctx, dy):
        from llm_research_b200.ops.gemm import linear_dgrad

        x, w = ctx.saved_tensors
        comm, group = ctx.comm, ctx.group
        dy = dy.contiguous()
        T = dy.shape[0] * dist.get_world_size(group)
        dres = dy if ctx.has_residual else None
        if _fused_ok(comm, dy, T, (w.shape[0], w.shape[1])):
            dx, dy_full = comm.ag_gemm(dy, w.t().contiguous())
        else:
            dy_full = _gather_rows(dy, comm, group)
            dx = linear_dgrad(dy_full, w)
        dw = _wgrad(dy_full, x, w) if ctx.needs_input_grad[1] else None
        return dx, dw, dres, None, None


class ColumnParallelLinear(nn.Module):
    """``(T/tp, in) -> (T, out/tp)``; weight shard ``(out/tp, in)``."""

    def __init__(self, in_features: int, out_features: int, group: Optional[dist.ProcessGroup] = None,
                 comm: Optional[TPComm] = None, device=None, dtype=None) -> None:
        super().__init__()
        self.group, self.comm = group, comm
        tp = dist.get_world_size(group)
        assert out_features % tp == 0
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features // tp, in_features, device=device, dtype=dtype))
        nn.init.normal_(self.weight, std=0.02)

    def forward(self, x_shard: torch.Tensor) -> torch.Tensor:
        return column_parallel(x_shard, self.weight, self.group, self.comm)


class RowParallelLinear(nn.Module):
    """``(T, in/tp) -> (T/tp, out)`` (+ residual); weight shard ``(out, in/tp)``."""

    def __init__(self, in_features: int, out_features: int, group: Optional[dist.ProcessGroup] = None,
                 comm: Optional[TPComm] = None, device=None, dtype=None) -> None:
        super().__init__()
        self.group, self.comm = group, comm
        tp = dist.get_world_size(group)
        assert in_features % tp == 0
        self.in_features, self.out_features = in_features, out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features // tp, device=device, dtype=dtype))
        nn.init.normal_(self.weight, std=0.02 / math.sqrt(2.0))

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        return row_parallel(x, self.weight, self.group, self.comm, residual)


def shard_linear_weight(w: torch.Tensor, group: Optional[dist.ProcessGroup], dim: int) -> torch.Tensor:
    """This rank's slice of a full weight: ``dim=0`` for column parallel, ``1`` for row parallel."""
    tp, r = dist.get_world_size(group), dist.get_rank(group)
    return w.chunk(tp, dim=dim)[r].contiguous()


# ----------------------------------------------------------- model integration
_TP_STATE: Optional[Tuple[dist.ProcessGroup, Optional[TPComm]]] = None


@contextlib.contextmanager
def tensor_parallel(group: dist.ProcessGroup, comm: Optional[TPComm] = None):
    """Modules built inside this context (Tier-1 attention and SwiGLU FFN) hold
    their ``1/tp`` weight shards and run sequence-parallel over ``group``;
    ``comm`` (a :class:`TPComm`) selects the fused symmetric-memory kernels,
    ``None`` the NCCL collectives."""
    global _TP_STATE
    prev = _TP_STATE
    _TP_STATE = (group, comm)
    try:
        yield
    finally:
        _TP_STATE = prev


_TP_SCOPE = False


@contextlib.contextmanager
def tensor_parallel_scope():
    """Opened by the Tier-1 trunk while it builds its blocks: only modules built
    inside it are split (the tiers after Tier 1 run replicated)."""
    global _TP_SCOPE
    prev = _TP_SCOPE
    _TP_SCOPE = True
    try:
        yield
    finally:
        _TP_SCOPE = prev


def current_tensor_parallel() -> Optional[Tuple[dist.ProcessGroup, Optional[TPComm]]]:
    return _TP_STATE if _TP_SCOPE else None


def enclosing_tensor_parallel_group() -> Optional[dist.ProcessGroup]:
    """The group of an enclosing ``tensor_parallel`` context with more than one
    rank, inside or outside the trunk's scope (the head uses it for the
    vocabulary-parallel loss); ``None`` otherwise."""
    if _TP_STATE is None or dist.get_world_size(_TP_STATE[0]) < 2:
        return None
    return _TP_STATE[0]


def mark_tp(p: nn.Parameter, dim: int) -> nn.Parameter:
    """Tag a TP weight shard with the dimension along which the shards of the
    group concatenate to the full weight (0: column parallel, 1: row parallel)."""
    p._lrb_tp = dim
    return p


class _ScatterSeq(torch.autograd.Function):
    """Replicated ``(T, d)`` -> this rank's contiguous ``T/tp`` rows; backward all-gathers."""

    @staticmethod
    def forward(ctx, x2d, group):
        ctx.group = group
        W, r = dist.get_world_size(group), dist.get_rank(group)
        n = x2d.shape[0] // W
        return x2d[r * n:(r + 1) * n].clone()

    @staticmethod
    def backward(ctx, g):
        return _all_gather_rows(g.contiguous(), ctx.group), None


class _GatherSeq(torch.autograd.Function):
    """Sequence shards ``(T/tp, d)`` -> replicated ``(T, d)``; the computation that
    follows is replicated on every rank, so backward keeps this rank's rows."""

    @staticmethod
    def forward(ctx, x_shard, group):
        ctx.group = group
        return _all_gather_rows(x_shard, group)

    @staticmethod
    def backward(ctx, g):
        W, r = dist.get_world_size(ctx.group), dist.get_rank(ctx.group)
        n = g.shape[0] // W
        return g[r * n:(r + 1) * n].contiguous(), None


class _SumGrad(torch.autograd.Function):
    """Identity whose backward sums the gradient over the group: a weight that is
    replicated but applied to sequence shards (the block norms) gets the full gradient."""

    @staticmethod
    def forward(ctx, w, group):
        ctx.group = group
        return w.view_as(w)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g, None


def scatter_sequence(x: torch.Tensor, group) -> torch.Tensor:
    """``(B, S, d)`` replicated -> ``(B*S/tp, d)`` sequence shard (flattened token order)."""
    return _ScatterSeq.apply(x.reshape(-1, x.shape[-1]), group)


def gather_sequence(x_shard: torch.Tensor, group, shape) -> torch.Tensor:
    return _GatherSeq.apply(x_shard, group).view(shape)


def sum_grad(w: torch.Tensor, group) -> torch.Tensor:
    return _SumGrad.apply(w, group)


def column_parallel(x_shard: torch.Tensor, w: torch.Tensor, group, comm: Optional[TPComm]) -> torch.Tensor:
    """``(T/tp, in) -> (T, out/tp)``: the fused kernels in bf16, else ``project`` after
    a differentiable row all-gather (NVFP4 GEMMs under NVFP4 precision)."""
    T = x_shard.shape[0] * dist.get_world_size(group)
    if _fused_ok(comm, x_shard, T, (x_shard.shape[1], w.shape[0])):
        return _ColumnFn.apply(x_shard, w, comm, group)
    return project(_AllGatherRows.apply(x_shard, comm, group), w)


def row_parallel(x: torch.Tensor, w: torch.Tensor, group, comm: Optional[TPComm],
                 residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``(T, in/tp) -> (T/tp, out)`` (+ residual, added in the reduction)."""
    if _fused_ok(comm, x, x.shape[0], (w.shape[0], w.shape[1])):
        return _RowFn.apply(x, w, residual, comm, group)
    return _ReduceScatterRows.apply(project(x, w), residual, comm, group)
