"""Expert parallelism for the MoE FFN: E routed experts sharded over an EP
group (``E / world`` experts per rank) plus an optional shared expert.

Per layer (``T`` tokens per rank, top-``k`` routing, capacity
``cap = ceil(capacity_factor * T * k / E)`` assignments per expert and source
rank, lowest (token, k) first):

1. router: fused softmax + top-k (``ops.softmax_topk``) -> weights, experts;
2. dispatch: each assignment's token row goes to its expert's owner, into
   slot ``[local expert][source rank][position]`` of the owner's buffer;
3. experts: per local expert one contiguous ``(world * cap, d)`` block, two
   batched GEMMs with the SwiGLU between them;
4. combine: every source pulls its k rows back and sums them with the routing
   weights.

Transport: with a :class:`EPComm` (one node, CUDA) dispatch is the
``ep_push`` kernel (P2P stores straight into the owners' buffers) and
combine the ``ep_pull`` kernel (P2P loads fused with the weighted sum); the
backward runs the same two kernels the other way round (combine-backward
pushes ``w * dy``, dispatch-backward pulls and sums).  Owner-side ordering
uses epoch flags in the heap: ``ready`` / ``consumed`` for the pushed buffer,
``out-ready`` / ``out-read`` for the pulled one.  Otherwise (CPU ranks, or no
heap) the same layout is exchanged with ``all_to_all_single`` (the baseline).
"""

from __future__ import annotations

import contextlib
import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from llm_research_b200 import ops
from llm_research_b200._ext import native
from llm_research_b200.utils.nvtx import nvtx_fn


_EP_CONTEXT = None


@contextlib.contextmanager
def expert_parallel(group: Optional[dist.ProcessGroup], comm: Optional["EPComm"] = None):
    """Models built inside this context give their MoE FFNs expert parallelism
    over ``group`` (each rank allocates only its own experts)."""
    global _EP_CONTEXT
    old = _EP_CONTEXT
    _EP_CONTEXT = (group, comm)
    try:
        yield
    finally:
        _EP_CONTEXT = old


def current_expert_parallel():
    return _EP_CONTEXT


def make_route(idx: torch.Tensor, experts_per_rank: int, num_experts: int, cap: int, with_counts: bool = False):
    """``(dest, local_expert, slot)`` int32 per assignment (``slot = -1``: over
    capacity), and the per-expert assignment counts when ``with_counts``: one
    device kernel (``ops.route_slots``) on CUDA."""
    dest, le, slot, counts = ops.route_slots(idx, num_experts, experts_per_rank, cap)
    route = (dest.contiguous(), le.contiguous(), slot.contiguous())
    return (route, counts) if with_counts else route


class EPComm:
    def __init__(self, group: Optional[dist.ProcessGroup], max_tokens: int, top_k: int, d: int,
                 experts_per_rank: int, capacity_factor: float, device: torch.device) -> None:
        from llm_research_b200.parallel.symm import SymmetricHeap

        self.group = group
        self.world = W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.epl, self.d, self.device = experts_per_rank, d, device
        E = W * experts_per_rank
        self.cap_max = math.ceil(capacity_factor * max_tokens * top_k / E)
        region = experts_per_rank * W * self.cap_max * d * 2
        self.heap = h = SymmetricHeap(2 * region + 8192, group=group, device=device)
        self.recv_off, self.out_off = h.alloc(region), h.alloc(region)
        self.ready_off, self.consumed_off = h.alloc(4 * W), h.alloc(4)
        self.outready_off, self.outread_off = h.alloc(4), h.alloc(4 * W)
        self.ready = h.view(self.ready_off, (W,), torch.int32)
        self.consumed = h.view(self.consumed_off, (1,), torch.int32)
        self.outready = h.view(self.outready_off, (1,), torch.int32)
        self.outread = h.view(self.outread_off, (W,), torch.int32)
        self.counters = torch.zeros(4, dtype=torch.int32, device=device)
        self.eR = 0
        self.eO = 0

    def _region(self, off: int, cap: int) -> torch.Tensor:
        return self.heap.view(off, (self.epl, self.world * cap, self.d), torch.bfloat16)

    # pushed channel (sources -> owners)
    @nvtx_fn("lrb/ep/dispatch_push")
    def push(self, rows: torch.Tensor, scale: Optional[torch.Tensor], per_assignment: bool, route, cap: int, k: int):
        self.eR += 1
        native().ep_push(rows.contiguous(), scale, per_assignment, self.heap.bases, self.recv_off, self.ready_off,
                         self.consumed_off, self.rank, self.world, k, cap, self.epl, self.eR, *route,
                         self.counters[0:1], self.heap.err)

    @nvtx_fn("lrb/ep/dispatch_take")
    def take(self, cap: int) -> torch.Tensor:
        C = native()
        C.ep_flag_wait(self.ready, self.world, self.eR, self.heap.err)
        region = self._region(self.recv_off, cap)
        out = region.clone()
        region.zero_()  # unused slots must read as zeros next time
        C.ep_flag_set(self.consumed, self.eR)
        return out

    # pulled channel (owners -> sources)
    @nvtx_fn("lrb/ep/combine_put")
    def put(self, t: torch.Tensor, cap: int) -> None:
        C = native()
        self.eO += 1
        C.ep_flag_wait(self.outread, self.world, self.eO - 1, self.heap.err)
        self._region(self.out_off, cap).copy_(t)
        C.ep_flag_set(self.outready, self.eO)

    @nvtx_fn("lrb/ep/combine_pull")
    def pull(self, T: int, w: Optional[torch.Tensor], want_rows: bool, route, cap: int, k: int):
        y = torch.empty(T, self.d, dtype=torch.bfloat16, device=self.device)
        rows = torch.empty(T * k, self.d, dtype=torch.bfloat16, device=self.device) if want_rows else None
        native().ep_pull(y, rows, w, self.heap.bases, self.out_off, self.outready_off, self.outread_off, self.rank,
                         self.world, k, cap, self.epl, self.eO, *route, self.counters[1:2], self.heap.err)
        return y, rows

    def close(self) -> None:
        self.heap.close()


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm, route, cap, k):
        ctx.comm, ctx.route, ctx.cap, ctx.k, ctx.T = comm, route, cap, k, x.shape[0]
        comm.push(x, None, False, route, cap, k)
        return comm.take(cap)

    @staticmethod
    def backward(ctx, g_xe):
        comm = ctx.comm
        comm.put(g_xe.contiguous().to(torch.bfloat16), ctx.cap)
        gx, _ = comm.pull(ctx.T, None, False, ctx.route, ctx.cap, ctx.k)
        return gx, None, None, None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y_e, w, comm, route, cap, k):
        T = w.shape[0]
        comm.put(y_e.contiguous().to(torch.bfloat16), cap)
        wf = w.reshape(-1).float().contiguous()
        y, rows = comm.pull(T, wf, True, route, cap, k)
        ctx.comm, ctx.route, ctx.cap, ctx.k = comm, route, cap, k
        ctx.save_for_backward(rows, wf)
        return y

    @staticmethod
    def backward(ctx, gy):
        rows, wf = ctx.saved_tensors
        comm, k = ctx.comm, ctx.k
        T = gy.shape[0]
        gy = gy.contiguous().to(torch.bfloat16)
        gw = (rows.view(T, k, -1).float() * gy.float()[:, None, :]).sum(-1)
        comm.push(gy, wf, False, ctx.route, ctx.cap, k)  # row t scaled by w[t, j] -> owner slot
        g_ye = comm.take(ctx.cap)
        return g_ye, gw, None, None, None, None


def _dispatch_collective(x, route, cap, world, epl, group):
    dest, le, slot = (r.long() for r in route)
    T, d = x.shape
    k = dest.numel() // T
    valid = slot >= 0
    tok = torch.arange(dest.numel(), device=x.device) // k
    pos = (dest * epl + le) * cap + slot
    send = x.new_zeros(world * epl * cap, d)
    send = send.index_put((pos[valid],), x[tok[valid]], accumulate=False)
    from torch.distributed.nn.functional import all_to_all_single

    recv = all_to_all_single(torch.empty_like(send), send, group=group)
    return recv.view(world, epl, cap, d).permute(1, 0, 2, 3).reshape(epl, world * cap, d)


def _combine_collective(y_e, w, route, cap, world, epl, group):
    dest, le, slot = (r.long() for r in route)
    d = y_e.shape[-1]
    send = y_e.reshape(epl, world, cap, d).permute(1, 0, 2, 3).reshape(world * epl * cap, d)
    from torch.distributed.nn.functional import all_to_all_single

    back = all_to_all_single(torch.empty_like(send), send, group=group)
    pos = ((dest * epl + le) * cap + slot.clamp(min=0))
    rows = back[pos] * (slot >= 0).to(back.dtype)[:, None]
    T = w.shape[0]
    return (rows.view(T, -1, d) * w.to(rows.dtype)[..., None]).sum(1)


class ExpertParallelMoE(nn.Module):
    """SwiGLU MoE with E experts over the EP group (+ an optional shared expert)."""

    def __init__(self, d_model: int, d_ff: int, num_experts: int, top_k: int = 2, capacity_factor: float = 1.25,
                 group: Optional[dist.ProcessGroup] = None, shared_expert: bool = True,
                 comm: Optional[EPComm] = None, device=None, dtype=None) -> None:
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert num_experts % self.world == 0
        self.epl = num_experts // self.world
        self.num_experts, self.top_k, self.capacity_factor = num_experts, top_k, capacity_factor
        self.d_model, self.d_ff = d_model, d_ff
        self.comm = comm
        self.router = nn.Linear(d_model, num_experts, bias=False, device=device, dtype=dtype)
        self.w_up_gate = nn.Parameter(torch.empty(self.epl, 2 * d_ff, d_model, device=device, dtype=dtype))
        self.w_down = nn.Parameter(torch.empty(self.epl, d_model, d_ff, device=device, dtype=dtype))
        nn.init.normal_(self.router.weight, std=0.02)
        nn.init.normal_(self.w_up_gate, std=0.02)
        nn.init.normal_(self.w_down, std=0.02 / math.sqrt(2.0))
        # this rank's experts: not sharded or reduced by the data-parallel engine
        self.w_up_gate._lrb_local = True
        self.w_down._lrb_local = True
        self.shared = None
        if shared_expert:
            from genesis.model.ffn import SwiGLUFFN

            self.shared = SwiGLUFFN(d_model=d_model, d_ff=d_ff).to(device=device, dtype=dtype)
        self.last_aux: Optional[torch.Tensor] = None

    def experts(self, x_e: torch.Tensor) -> torch.Tensor:
        """This rank's experts on their dispatch rows ``(epl, rows, d)``: batched
        CTA-pair GEMMs over the expert dimension (``ops.linear.grouped_swiglu``)."""
        from llm_research_b200.ops.linear import grouped_swiglu

        return grouped_swiglu(x_e, self.w_up_gate.to(x_e.dtype), self.w_down.to(x_e.dtype))

    def load_balance_loss(self) -> torch.Tensor:
        return self.last_aux if self.last_aux is not None else torch.zeros((), device=self.router.weight.device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        T = xf.shape[0]
        from llm_research_b200.ops.linear import dense

        logits = dense(xf, self.router.weight)  # the pair GEMM where it applies
        w, idx, probs = ops.softmax_topk(logits.float(), self.top_k)
        cap = math.ceil(self.capacity_factor * T * self.top_k / self.num_experts)
        route, counts = make_route(idx, self.epl, self.num_experts, cap, with_counts=True)
        # Switch-style load balance: E * sum_e fraction_e * mean_prob_e, the
        # fractions from the routing kernel's per-expert counts
        frac = counts.float() / max(T * self.top_k, 1)
        self.last_aux = self.num_experts * (frac * probs.mean(0)).sum()
        fused = self.comm is not None and xf.is_cuda and xf.dtype == torch.bfloat16 and cap <= self.comm.cap_max
        if fused:
            x_e = _Dispatch.apply(xf, self.comm, route, cap, self.top_k)
            y = _Combine.apply(self.experts(x_e), w, self.comm, route, cap, self.top_k)
        else:
            x_e = _dispatch_collective(xf, route, cap, self.world, self.epl, self.group)
            y = _combine_collective(self.experts(x_e), w, route, cap, self.world, self.epl, self.group)
        if self.shared is not None:
            y = y + self.shared(xf)
        return y.reshape(shape)
