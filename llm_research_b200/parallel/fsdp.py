"""Flat-parameter fully sharded data parallel engine (ZeRO-3 style) with
mixed precision, used for every training run including a single GPU.

Layout.  Parameters are grouped into *units*: every transformer block is one
unit, everything else (embeddings, gates, pooling, norms, ...) forms the root
unit.  Each unit owns

* a flat bf16 compute buffer (full size while gathered; its storage is freed
  between uses when ``reshard_after_forward``) whose views are handed to the
  module through ``torch.func.functional_call``;
* a flat fp32 gradient accumulator (local, full size) that the backward of
  every weight view adds into, so micro-step accumulation happens in fp32;
* this rank's shard of the fp32 master weights, of the reduced gradient and
  of the optimizer state (``numel / world`` elements each, 8-element aligned).

Step flow.  Before a unit's forward (and again before its backward) its bf16
shards are all-gathered into the compute buffer on a communication stream,
one unit ahead of use.  When the last gradient of a unit has been
accumulated on the boundary micro-step, the unit's fp32 gradient is
reduce-scattered into the shard.  The optimizer (:class:`ShardedHybridOptimizer`)
then updates the shards; Muon matrices are gathered to an owner rank for the
Newton-Schulz iteration and the scaled update is scattered back (distributed
Muon), so Muon always sees whole 2-D matrices -- unlike the reference, whose
FSDP1 flattening routes every parameter to AdamW
(``olympus/distributed/fsdp_wrapper.py:149`` with
``olympus/optim/muon_adamw_hybrid.py:113-116``).

With ``world_size == 1`` the same code runs without collectives: the master
buffer is the whole model and ``refresh`` casts it into the compute buffer.

Collectives.  ``comm="nccl"`` issues NCCL all-gather / reduce-scatter on the
communication stream (the baseline).  ``comm="p2p"`` (one node) runs the
framework's own kernels on symmetric memory (:mod:`llm_research_b200.parallel.symm`):

* reduce-scatter = ``p2p_rs_push`` (each rank casts its fp32 accumulator to
  bf16, stores every owner's slice into that owner's receive slot over NVLink
  and zeroes the accumulator in the same pass) + ``p2p_rs_reduce`` (the owner
  sums the slots in fp32, scales by 1/world, writes the shard and adds the
  sum of squares used by gradient clipping -- no separate norm pass);
* all-gather = ``p2p_ag_publish`` (the optimizer's fp32 master shard is cast
  to bf16 straight into the heap) + ``p2p_pull`` (each rank reads all shards).

``comm="nvls"`` (one node with NVSwitch multicast) runs the kernels of
:mod:`llm_research_b200.parallel.nvls` on a multicast heap:

* reduce-scatter = ``nvls_rs_stage`` (the fp32 accumulator is cast to bf16
  into this rank's copy of a staging buffer and zeroed) + ``nvls_rs_reduce``
  (the owner reads its shard with ``multimem.ld_reduce``: the switch sums the
  ranks' copies in fp32; then scale, store and sum of squares as above);
* all-gather = ``nvls_ag_publish`` once per optimizer step, on the
  communication stream: every rank casts its master shard to bf16 and
  ``multimem.st`` writes it into its slot of every rank's gathered-parameter
  buffer, so the bf16 parameters stay resident and each gather reduces to one
  flag wait per unit and step.  Memory per rank: 2 bytes per parameter for the
  gathered copy plus 2 for the staging buffer (sharded fp32 master, gradient
  shard and optimizer state as in the other modes).  The publish first
  exchanges "released" flags so no rank overwrites weights a peer still reads.

Ordering argument for reusing the heap shard: a rank republishes a unit's
shard only after its reduce of that unit, which waited for every peer's push
of the unit, and each peer pushes only after its backward of the unit, which
came after its last pull of the unit.
"""

from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterator, List, Optional, Sequence, Set, Tuple, Type

import torch
import torch.distributed as dist
import torch.nn as nn

from llm_research_b200 import ops
from llm_research_b200.utils.nvtx import nvtx_fn

ALIGN = 8  # elements; keeps every bf16 view 16-byte aligned


def ops_native():
    from llm_research_b200._ext import native

    return native()


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class ParamInfo:
    name: str
    param: nn.Parameter
    unit: int
    offset: int  # in the unit's flat buffer
    shape: Tuple[int, ...]
    numel: int
    index: int  # position in model.parameters() order (optimizer-state key)


@dataclass
class Unit:
    index: int
    module: nn.Module
    params: List[ParamInfo] = field(default_factory=list)
    total: int = 0      # padded flat size (multiple of world * ALIGN)
    shard: int = 0      # per-rank shard size
    compute: Optional[torch.Tensor] = None
    views: Dict[str, torch.Tensor] = field(default_factory=dict)
    grad_acc: Optional[torch.Tensor] = None
    master: Optional[torch.Tensor] = None
    grad_shard: Optional[torch.Tensor] = None
    compute_shard: Optional[torch.Tensor] = None
    writer: Optional[torch.Tensor] = None
    gathered: bool = False
    gather_event: Optional[torch.cuda.Event] = None
    pending_grads: int = 0
    grads_seen: Set[int] = field(default_factory=set)
    reduced: bool = False
    rs_event: Optional[torch.cuda.Event] = None


class _GradSink(torch.autograd.Function):
    """Identity on a compute-weight view; its gradient is added to the unit's
    fp32 accumulator instead of flowing to a leaf."""

    @staticmethod
    def forward(ctx, anchor, view, engine, unit_idx, pidx):
        ctx.engine = engine
        ctx.key = (unit_idx, pidx)
        return view.view_as(view)

    @staticmethod
    def backward(ctx, grad):
        from llm_research_b200.ops.linear import is_accumulated_marker

        # The marker means the producing GEMM already added this gradient into the
        # accumulator (see llm_research_b200.ops.linear): bookkeeping only.
        ctx.engine._accumulate(ctx.key[0], ctx.key[1], None if is_accumulated_marker(grad) else grad)
        return None, None, None, None, None


def default_unit_classes() -> Tuple[Type[nn.Module], ...]:
    from genesis.model.memory_layer import MemoryReadLayer
    from genesis.model.tier1_token_processor import TransformerBlock

    return (TransformerBlock, MemoryReadLayer)


class FlatShardEngine(nn.Module):
    """Wraps ``module``; call it like the module.  See the module docstring."""

    def __init__(
        self,
        module: nn.Module,
        process_group: Optional[dist.ProcessGroup] = None,
        compute_dtype: torch.dtype = torch.bfloat16,
        reshard_after_forward: bool = True,
        unit_classes: Optional[Sequence[Type[nn.Module]]] = None,
        device: Optional[torch.device] = None,
        reduce_dtype: torch.dtype = torch.float32,
        comm: Optional[str] = None,
        tp_group: Optional[dist.ProcessGroup] = None,
        replicate: bool = False,
    ) -> None:
        super().__init__()
        self.module = module
        self.pg = process_group
        # Tensor parallelism across another group: parameters tagged ``_lrb_tp`` are
        # this rank's shards of larger weights, the rest are replicated over it.
        self.tp_group = tp_group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(process_group) if self.distributed else 1
        self.rank = dist.get_rank(process_group) if self.distributed else 0
        # ``replicate``: every rank keeps the whole model and optimizer (one
        # shard per rank of a world of one) and the unit gradients are averaged
        # with an all-reduce over the group instead of reduce-scattered -- the
        # DDP-like NO_SHARD strategy.
        self.replicas = 1
        if replicate and self.world > 1:
            self.replicas, self.world, self.rank = self.world, 1, 0
        self.compute_dtype = compute_dtype
        self.reduce_dtype = reduce_dtype
        self.reshard_after_forward = reshard_after_forward and self.world > 1
        self.device = device or next(module.parameters()).device
        self._sync_grads = True
        self._touched: Set[int] = set()  # ParamInfo.index of parameters that received a gradient
        self._in_backward = False
        self._anchor = torch.zeros((), device=self.device, requires_grad=True)
        self.comm_stream = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        classes = tuple(unit_classes) if unit_classes is not None else default_unit_classes()
        self._build_units(classes)
        self._rep_ranges = self._replicated_ranges() if tp_group is not None else None
        self._register_hooks()
        import os

        # Default: the own P2P gather / reduce-scatter on a single node of up to 4
        # ranks (at 2 ranks its reduce-scatter measured 1.34x NCCL and the training
        # step 1.3 % faster), NCCL above that (at 8 ranks NCCL's in-switch
        # reduction measured ahead, 0.95x for the P2P reduce-scatter).
        self.comm = (comm or os.environ.get("LRB_FSDP_COMM", "auto")).lower()
        if self.comm == "auto":
            self.comm = "p2p" if self.world <= 4 else "nccl"
        self.heap = None
        self._sumsq: Optional[torch.Tensor] = None
        if self.comm == "nvls":
            from llm_research_b200.parallel.nvls import NVLSUnavailable
            from llm_research_b200.parallel.symm import single_node

            if not (self.world > 1 and self.device.type == "cuda" and single_node(self.pg)):
                self.comm = "nccl"
            else:
                try:
                    self._setup_nvls()
                except NVLSUnavailable:
                    self.comm = "p2p"
        if self.comm == "p2p":
            from llm_research_b200.parallel.symm import single_node

            if not (self.world > 1 and self.device.type == "cuda" and single_node(self.pg)):
                self.comm = "nccl"
            else:
                self._setup_p2p()

    # ------------------------------------------------------------------ layout
    def _build_units(self, classes: Tuple[Type[nn.Module], ...]) -> None:
        unit_of_module: Dict[int, int] = {}
        self.units: List[Unit] = [Unit(index=0, module=self.module)]  # root
        # Exact type match: only blocks that run on every step become units,
        # so every rank issues the same collectives in the same order even
        # when data-dependent branches (HLRT tiers 2/3) differ between ranks.
        for m in self.module.modules():
            if m is not self.module and type(m) in classes:
                unit_of_module[id(m)] = len(self.units)
                self.units.append(Unit(index=len(self.units), module=m))
        owner: Dict[int, int] = {}
        for name, mod in self.module.named_modules():
            u = unit_of_module.get(id(mod))
            if u is not None:
                for pname, p in mod.named_parameters(recurse=True):
                    owner.setdefault(id(p), u)
        self.params: List[ParamInfo] = []
        # Rank-local parameters (expert-parallel experts, marked ``_lrb_local``)
        # are not sharded: they stay ordinary parameters whose gradients autograd
        # accumulates in ``.grad``; the optimizer steps them on their rank.
        self.local_params: List[Tuple[str, nn.Parameter]] = []
        seen: Set[int] = set()
        for idx, (name, p) in enumerate(self.module.named_parameters()):
            if id(p) in seen:
                continue
            seen.add(id(p))
            if getattr(p, "_lrb_local", False):
                self.local_params.append((name, p))
                continue
            u = self.units[owner.get(id(p), 0)]
            info = ParamInfo(name=name, param=p, unit=u.index, offset=u.total, shape=tuple(p.shape),
                             numel=p.numel(), index=len(self.params))
            u.params.append(info)
            u.total = _round_up(u.total + p.numel(), ALIGN)
            self.params.append(info)
        dev = self.device
        for u in self.units:
            u.total = _round_up(max(u.total, 1), self.world * ALIGN)
            u.shard = u.total // self.world
            full = torch.zeros(u.total, dtype=torch.float32, device=dev)
            for info in u.params:
                full[info.offset: info.offset + info.numel].copy_(info.param.detach().reshape(-1).float())
            lo = self.rank * u.shard
            u.master = full[lo: lo + u.shard].clone() if self.world > 1 else full
            u.grad_acc = torch.zeros(u.total, dtype=torch.float32, device=dev)
            u.grad_shard = torch.zeros(u.shard, dtype=torch.float32, device=dev) if self.world > 1 else u.grad_acc
            u.compute = torch.empty(u.total, dtype=self.compute_dtype, device=dev)
            # Writer alias of the same storage with its own version counter:
            # gathers and refreshes go through it, so autograd does not see
            # the re-materialisation of weights it saved for the backward.
            u.writer = torch.empty(0, dtype=self.compute_dtype, device=dev).set_(
                u.compute.untyped_storage(), 0, (u.total,), (1,))
            u.compute_shard = u.master.to(self.compute_dtype) if self.world > 1 else None
            for info in u.params:
                u.views[info.name] = u.compute[info.offset: info.offset + info.numel].view(info.shape)
            if self.world == 1:
                u.writer.copy_(u.master)
                u.gathered = True
                # The module's parameters alias the master weights.
                for info in u.params:
                    info.param.data = u.master[info.offset: info.offset + info.numel].view(info.shape)
            else:
                for info in u.params:
                    info.param.data = torch.empty(0, dtype=torch.float32, device=dev)
                self._free(u)
            del full
        self.unit_order = [u.index for u in self.units[1:]]

    def _replicated_ranges(self) -> List[Tuple[int, int, int]]:
        """(unit, lo, hi) spans of this rank's grad shards that hold parameters not
        tagged ``_lrb_tp`` (replicated over the tensor-parallel group); merged."""
        out: List[Tuple[int, int, int]] = []
        for u in self.units:
            lo_s, hi_s = (self.rank * u.shard, (self.rank + 1) * u.shard) if self.world > 1 else (0, u.total)
            for info in u.params:
                if getattr(info.param, "_lrb_tp", None) is not None:
                    continue
                lo, hi = max(info.offset, lo_s), min(info.offset + info.numel, hi_s)
                if lo >= hi:
                    continue
                lo, hi = lo - lo_s, hi - lo_s
                if out and out[-1][0] == u.index and out[-1][2] == lo:
                    out[-1] = (u.index, out[-1][1], hi)
                else:
                    out.append((u.index, lo, hi))
        return out

    # ------------------------------------------------------------ p2p comm
    def _setup_p2p(self) -> None:
        from llm_research_b200.parallel.symm import SymmetricHeap

        W = self.world
        need = 0
        for u in self.units:
            need += _round_up(W * u.shard * 2, 256) + 256 * 4 + _round_up(u.shard * 2, 256)
        self.heap = heap = SymmetricHeap(need + (1 << 20), group=self.pg, device=self.device)
        for u in self.units:
            u.recv_off = heap.alloc(W * u.shard * 2)
            u.ready_off = heap.alloc(4 * W)
            u.consumed_off = heap.alloc(4)
            u.ag_off = heap.alloc(u.shard * 2)
            u.agready_off = heap.alloc(4)
            u.recv = heap.view(u.recv_off, (W * u.shard,), torch.bfloat16)
            u.ready = heap.view(u.ready_off, (W,), torch.int32)
            u.consumed = heap.view(u.consumed_off, (1,), torch.int32)
            u.agready = heap.view(u.agready_off, (1,), torch.int32)
            u.compute_shard = heap.view(u.ag_off, (u.shard,), torch.bfloat16)
            u.counters = torch.zeros(4, dtype=torch.int32, device=self.device)
            u.rs_epoch = 0
        self._sumsq = torch.zeros((), dtype=torch.float32, device=self.device)
        self._ag_epoch = 0
        dist.barrier(group=self.pg)  # every heap is zeroed before anyone publishes
        self._publish()

    def _setup_nvls(self) -> None:
        from llm_research_b200.parallel.nvls import MulticastHeap

        W = self.world
        need = sum(2 * _round_up(u.total * 2, 256) + _round_up(16 * W, 256) for u in self.units)
        self.heap = heap = MulticastHeap(need + (1 << 20), group=self.pg, device=self.device)
        for u in self.units:
            u.nv_ag_off = heap.alloc(u.total * 2)
            u.nv_stage_off = heap.alloc(u.total * 2)
            u.nv_flag_off = heap.alloc(16 * W)
            u.nv_stage = heap.view(u.nv_stage_off, (u.total,), torch.bfloat16)
            flags = heap.view(u.nv_flag_off, (4 * W,), torch.int32)
            # ready[W] and consumed[W] of the reduce-scatter, released[W] and
            # published[W] of the all-gather; peer r writes entry r.
            u.nv_ready, u.nv_consumed, u.nv_agfree, u.nv_agready = (flags[i * W:(i + 1) * W] for i in range(4))
            u.nv_seen = 0
            # The gathered bf16 parameters live in the heap for good: the compute
            # buffer, its writer alias and the weight views all point there.
            u.compute = heap.view(u.nv_ag_off, (u.total,), self.compute_dtype)
            u.writer = torch.empty(0, dtype=self.compute_dtype, device=self.device).set_(
                u.compute.untyped_storage(), u.compute.storage_offset(), (u.total,), (1,))
            for info in u.params:
                u.views[info.name] = u.compute[info.offset: info.offset + info.numel].view(info.shape)
            u.counters = torch.zeros(4, dtype=torch.int32, device=self.device)
            u.rs_epoch = 0
            u.gathered = False
        self._sumsq = torch.zeros((), dtype=torch.float32, device=self.device)
        self._ag_epoch = 0
        self._publish()

    @nvtx_fn("lrb/fsdp/publish")
    def _publish(self) -> None:
        C = ops_native()
        self._ag_epoch += 1
        if self.comm == "nvls":
            # On the communication stream, after the optimizer step: the next
            # forward's units wait for their own broadcast only (``_gather``), so
            # the broadcast of later units overlaps the compute of earlier ones.
            h, W = self.heap, self.world
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm_stream):
                for u in self.units:
                    C.nvls_ag_publish(u.master, h.mc(u.nv_ag_off), u.nv_agfree, h.bases, u.nv_flag_off + 8 * W,
                                      u.nv_flag_off + 12 * W, self.rank, W, self._ag_epoch, u.counters[2:3], h.err)
            return
        for u in self.units:
            C.p2p_ag_publish(u.master, u.compute_shard, u.agready, self._ag_epoch, u.counters[2:3])

    def close(self) -> None:
        """Release the symmetric heap (collective)."""
        if self.heap is not None:
            self.heap.close()
            self.heap = None

    # --------------------------------------------------------------- gathers
    def _free(self, u: Unit) -> None:
        if getattr(self, "comm", None) == "nvls":  # resident in the multicast heap
            return
        if self.world > 1 and u.compute.untyped_storage().size() > 0:
            u.compute.untyped_storage().resize_(0)
        u.gathered = self.world == 1

    @nvtx_fn("lrb/fsdp/ag")
    def _gather(self, u: Unit, wait: bool = True) -> None:
        if self.world == 1:
            return
        if not u.gathered and self.comm_stream is None:  # CPU ranks (gloo): synchronous
            st = u.compute.untyped_storage()
            if st.size() == 0:
                st.resize_(u.total * u.compute.element_size())
            dist.all_gather_into_tensor(u.writer, u.compute_shard, group=self.pg)
            u.gathered = True
            return
        if self.comm == "nvls":
            # The publish after the optimizer step already broadcast the shards:
            # wait (once per step) for every rank's flag of this unit.
            if u.nv_seen != self._ag_epoch:
                self.comm_stream.wait_stream(torch.cuda.current_stream(self.device))
                with torch.cuda.stream(self.comm_stream):
                    ops_native().nvls_wait(u.nv_agready, self.world, self._ag_epoch, self.heap.err)
                    ev = torch.cuda.Event()
                    ev.record(self.comm_stream)
                u.gather_event = ev
                u.nv_seen = self._ag_epoch
            u.gathered = True
            if wait and u.gather_event is not None:
                self._wait_comm(u.gather_event)
                u.gather_event = None
            return
        if not u.gathered:
            st = u.compute.untyped_storage()
            if st.size() == 0:
                st.resize_(u.total * u.compute.element_size())
            cur = torch.cuda.current_stream(self.device)
            self.comm_stream.wait_stream(cur)
            with torch.cuda.stream(self.comm_stream):
                if self.heap is not None:
                    ops_native().p2p_pull(u.writer, self.heap.bases, u.ag_off, u.agready_off, self.world,
                                          self._ag_epoch, self.heap.err)
                else:
                    dist.all_gather_into_tensor(u.writer, u.compute_shard, group=self.pg)
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
            u.gather_event = ev
            u.gathered = True
        if wait and u.gather_event is not None:
            self._wait_comm(u.gather_event)
            u.gather_event = None

    # ----------------------------------------------------- exposed communication
    _exposed_pairs: Optional[List[Tuple[torch.cuda.Event, torch.cuda.Event]]] = None

    def _wait_comm(self, ev: torch.cuda.Event) -> None:
        """Make the compute stream wait for a communication event; when measuring,
        bracket the wait with events so the stall can be timed on the device."""
        cur = torch.cuda.current_stream(self.device)
        if self._exposed_pairs is None:
            cur.wait_event(ev)
            return
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        cur.wait_event(ev)
        e1.record(cur)
        self._exposed_pairs.append((e0, e1))

    def start_exposed_comm_measurement(self) -> None:
        self._exposed_pairs = []

    def stop_exposed_comm_measurement(self) -> float:
        """Milliseconds the compute stream spent waiting for communication since
        ``start_exposed_comm_measurement`` (synchronises the device)."""
        pairs, self._exposed_pairs = self._exposed_pairs or [], None
        torch.cuda.synchronize(self.device)
        return float(sum(a.elapsed_time(b) for a, b in pairs))

    def _prefetch(self, pos: int) -> None:
        if 0 <= pos < len(self.unit_order):
            self._gather(self.units[self.unit_order[pos]], wait=False)

    # ----------------------------------------------------------------- hooks
    def _register_hooks(self) -> None:
        self._pos = {ui: i for i, ui in enumerate(self.unit_order)}
        for ui in self.unit_order:
            u = self.units[ui]
            u.module.register_forward_pre_hook(self._make_pre_forward(ui))
            u.module.register_forward_hook(self._make_post_forward(ui))

    def _make_pre_forward(self, ui: int):
        def hook(module, args):
            if not self._active:
                return
            self._gather(self.units[ui], wait=True)
            self._prefetch(self._pos[ui] + 1)
        return hook

    def _make_post_forward(self, ui: int):
        def hook(module, args, output):
            if not self._active:
                return
            if self.reshard_after_forward:
                self._free(self.units[ui])
            if torch.is_grad_enabled() and isinstance(output, torch.Tensor) and output.requires_grad:
                output.register_hook(self._make_pre_backward(ui))
        return hook

    def _make_pre_backward(self, ui: int):
        def hook(grad):
            self._begin_backward()
            self._gather(self.units[ui], wait=True)
            self._prefetch(self._pos[ui] - 1)
            return grad
        return hook

    def _begin_backward(self) -> None:
        if not self._in_backward:
            self._in_backward = True
            torch.autograd.Variable._execution_engine.queue_callback(self._end_backward)

    # ---------------------------------------------------------- grad plumbing
    def _accumulate(self, ui: int, pidx: int, grad: torch.Tensor) -> None:
        self._begin_backward()
        u = self.units[ui]
        info = u.params[pidx]
        if grad is not None:
            dst = u.grad_acc[info.offset: info.offset + info.numel].view(info.shape)
            dst.add_(grad)  # bf16 -> fp32 accumulate in one pass (no separate cast)
        u.grads_seen.add(pidx)
        self._touched.add(info.index)
        if len(u.grads_seen) == len(u.params):
            self._unit_backward_done(u)

    def _unit_backward_done(self, u: Unit, final: bool = False) -> None:
        # The root unit is only completed at the end of backward (its
        # parameters may belong to branches some ranks skip).
        if u.reduced or (u.index == 0 and not final):
            return
        u.reduced = True
        if u.index != 0 and self.world > 1:
            self._free(u)
        if self._sync_grads:
            self._reduce_scatter(u)

    @nvtx_fn("lrb/fsdp/rs")
    def _reduce_scatter(self, u: Unit) -> None:
        if self.world == 1:
            if self.replicas > 1:
                self._all_reduce(u)
            return
        if self.comm_stream is None:
            dist.reduce_scatter_tensor(u.grad_shard, u.grad_acc, op=dist.ReduceOp.AVG, group=self.pg)
            u.grad_acc.zero_()
            return
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        if self.comm == "nvls":
            C, h, W = ops_native(), self.heap, self.world
            u.rs_epoch += 1
            with torch.cuda.stream(self.comm_stream):
                C.nvls_rs_stage(u.grad_acc, u.nv_stage, u.nv_consumed, h.bases, u.nv_flag_off, self.rank, W,
                                u.rs_epoch, u.counters[0:1], h.err)
                C.nvls_rs_reduce(h.mc(u.nv_stage_off), u.grad_shard, 1.0 / W, False, u.nv_ready, h.bases,
                                 u.nv_flag_off + 4 * W, self.rank, W, u.rs_epoch, self._sumsq, u.counters[1:2],
                                 h.err)
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
            u.rs_event = ev
            return
        if self.heap is not None:
            C = ops_native()
            u.rs_epoch += 1
            with torch.cuda.stream(self.comm_stream):
                C.p2p_rs_push(u.grad_acc, self.heap.bases, u.recv_off, u.ready_off, u.consumed_off, self.rank,
                              self.world, u.shard, u.rs_epoch, u.counters[0:1], self.heap.err)
                C.p2p_rs_reduce(u.recv, u.grad_shard, self.world, 1.0 / self.world, False, u.ready, u.consumed,
                                u.rs_epoch, self._sumsq, u.counters[1:2], self.heap.err)
                ev = torch.cuda.Event()
                ev.record(self.comm_stream)
            u.rs_event = ev
            return
        with torch.cuda.stream(self.comm_stream):
            src = u.grad_acc if self.reduce_dtype == torch.float32 else u.grad_acc.to(self.reduce_dtype)
            out = u.grad_shard if self.reduce_dtype == torch.float32 else torch.empty(u.shard, dtype=self.reduce_dtype, device=self.device)
            dist.reduce_scatter_tensor(out, src, op=dist.ReduceOp.AVG, group=self.pg)
            if out is not u.grad_shard:
                u.grad_shard.copy_(out)
            u.grad_acc.zero_()
            ev = torch.cuda.Event()
            ev.record(self.comm_stream)
        u.rs_event = ev

    def _all_reduce(self, u: Unit) -> None:
        """Replicated parameters: average the unit's fp32 gradient over the group
        in place (sum, then 1/replicas: gloo has no average)."""
        if self.comm_stream is None:
            dist.all_reduce(u.grad_acc, group=self.pg)
            u.grad_acc.mul_(1.0 / self.replicas)
            return
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            dist.all_reduce(u.grad_acc, group=self.pg)
            u.grad_acc.mul_(1.0 / self.replicas)
            ev = torch.cuda.Event()
            ev.record(self.comm_stream)
        u.rs_event = ev

    def _end_backward(self) -> None:
        # Units whose parameters did not all receive gradients (unused
        # branches) are completed here.
        for u in self.units:
            self._unit_backward_done(u, final=True)
        if self.world > 1:
            self._free(self.units[0])
        for u in self.units:
            u.grads_seen.clear()
            u.reduced = False
        self._in_backward = False

    def wait_grads(self) -> None:
        """Make the current stream wait for every pending reduce-scatter."""
        if self.device.type != "cuda":
            return
        cur = torch.cuda.current_stream(self.device)
        for u in self.units:
            if u.rs_event is not None:
                self._wait_comm(u.rs_event)
                u.rs_event = None

    # ---------------------------------------------------------------- forward
    _active = False

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        self._gather(self.units[0], wait=True)
        tensors: Dict[str, torch.Tensor] = {}
        grad = torch.is_grad_enabled()
        for u in self.units:
            for pidx, info in enumerate(u.params):
                v = u.views[info.name]
                if grad:
                    t = _GradSink.apply(self._anchor, v, self, u.index, pidx)
                    # fp32 accumulator view: GEMMs that produce this weight's gradient
                    # may add into it directly (llm_research_b200.ops.linear)
                    t._lrb_acc = u.grad_acc[info.offset: info.offset + info.numel].view(info.shape)
                    tensors[info.name] = t
                else:
                    tensors[info.name] = v
        self._active = True
        try:
            out = torch.func.functional_call(self.module, tensors, args, kwargs, strict=False, tie_weights=True)
        finally:
            self._active = False
        return out

    @contextlib.contextmanager
    def no_sync(self) -> Iterator[None]:
        prev = self._sync_grads
        self._sync_grads = False
        try:
            yield
        finally:
            self._sync_grads = prev

    def set_sync(self, flag: bool) -> None:
        self._sync_grads = flag

    # ------------------------------------------------------------- utilities
    def grad_shards(self) -> List[torch.Tensor]:
        return [u.grad_shard for u in self.units]

    @torch.no_grad()
    @nvtx_fn("lrb/fsdp/clip")
    def clip_grad_norm_(self, max_norm: float, norm_type: float = 2.0) -> torch.Tensor:
        self.wait_grads()
        if self.heap is not None:
            sq = self._sumsq.clone()  # accumulated by the reduce kernels
        else:
            sq = torch.zeros((), dtype=torch.float32, device=self.device)
            for u in self.units:
                sq += u.grad_shard.float().pow(2).sum()
        local = [p.grad for _, p in self.local_params if p.grad is not None]
        for gr in local:  # disjoint per rank, like the shards: one sum over the group covers both
            sq += gr.float().pow(2).sum()
        if self._rep_ranges is not None:
            # Replicated parameters appear on every TP rank: count them once in the sum below.
            tp = dist.get_world_size(self.tp_group)
            rep = torch.zeros((), dtype=torch.float32, device=self.device)
            for ui, lo, hi in self._rep_ranges:
                rep += self.units[ui].grad_shard[lo:hi].float().pow(2).sum()
            sq = sq - (1.0 - 1.0 / tp) * rep
        if self.world > 1:
            dist.all_reduce(sq, group=self.pg)
        if self.tp_group is not None:
            dist.all_reduce(sq, group=self.tp_group)
        norm = sq.sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
        for u in self.units:
            u.grad_shard.mul_(coef)
        for gr in local:
            gr.mul_(coef.to(gr.dtype))
        return norm

    @torch.no_grad()
    def refresh(self) -> None:
        """Propagate updated master weights to the compute copies."""
        if self.heap is not None:
            self.heap.poll_error()
            self._publish()
            for u in self.units:
                self._free(u)
            return
        for u in self.units:
            if self.world == 1:
                u.writer.copy_(u.master)
            else:
                u.compute_shard.copy_(u.master)
                self._free(u)

    def touched_params(self, reduce_max: Optional[Callable[[torch.Tensor], torch.Tensor]] = None) -> Set[int]:
        """Parameters that received a gradient on any rank since ``zero_grad``
        (optimizers skip the others, like ``p.grad is None`` in torch).
        ``reduce_max``: the group-wide elementwise maximum to use instead of an
        all-reduce (the optimizer's symmetric-memory exchange)."""
        flags = torch.zeros(len(self.params), dtype=torch.float32, device=self.device)
        if self._touched:
            flags[list(self._touched)] = 1.0
        if reduce_max is not None and (self.world > 1 or self.replicas > 1):
            flags = reduce_max(flags)
        elif self.world > 1 or self.replicas > 1:
            dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.pg)
        return {i for i, f in enumerate(flags.tolist()) if f > 0}

    @torch.no_grad()
    def zero_grad(self) -> None:
        self._touched.clear()
        for _, p in self.local_params:
            p.grad = None
        if self._sumsq is not None:
            self._sumsq.zero_()
        for u in self.units:
            if self.world > 1:
                u.grad_shard.zero_()
            else:
                u.grad_acc.zero_()

    # ----------------------------------------------------------- checkpoints
    @torch.no_grad()
    def full_flat(self, u: Unit, src: torch.Tensor) -> torch.Tensor:
        """All-gather a per-unit shard-sized fp32 tensor into a full flat tensor."""
        if self.world == 1:
            return src
        out = torch.empty(u.total, dtype=src.dtype, device=self.device)
        dist.all_gather_into_tensor(out, src.contiguous(), group=self.pg)
        return out

    @torch.no_grad()
    def full_state_dict(self) -> Dict[str, torch.Tensor]:
        """Unsharded fp32 parameters by name (collective on every rank)."""
        out: Dict[str, torch.Tensor] = {}
        for u in self.units:
            full = self.full_flat(u, u.master)
            for info in u.params:
                out[info.name] = full[info.offset: info.offset + info.numel].view(info.shape).detach().cpu().clone()
        return out

    @torch.no_grad()
    def load_full_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        for u in self.units:
            full = torch.zeros(u.total, dtype=torch.float32, device=self.device)
            for info in u.params:
                if info.name in sd:
                    full[info.offset: info.offset + info.numel].copy_(sd[info.name].reshape(-1).float())
                else:
                    full[info.offset: info.offset + info.numel].copy_(self.full_flat(u, u.master)[info.offset: info.offset + info.numel])
            lo = self.rank * u.shard
            u.master.copy_(full[lo: lo + u.shard] if self.world > 1 else full)
        self.refresh()

    def make_optimizer(self, optimizer_cls: Type[torch.optim.Optimizer], defaults: Dict[str, Any]) -> "ShardedHybridOptimizer":
        from llm_research_b200.parallel.dmuon import ShardedHybridOptimizer

        return ShardedHybridOptimizer(self, optimizer_cls, defaults)
