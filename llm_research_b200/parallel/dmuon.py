"""Sharded optimizer for :class:`~llm_research_b200.parallel.fsdp.FlatShardEngine`,
including distributed Muon.

Each rank updates only its shard of every unit.  AdamW is elementwise and runs
directly on the shard (one multi-tensor launch).  Muon needs the whole matrix,
so for every Muon matrix an *owner* rank is chosen (greedy longest-processing-
time assignment by Newton-Schulz FLOPs, identical on all ranks) and:

1. every rank runs the fused prologue on the pieces it holds (decay,
   momentum, Nesterov direction in bf16, partial ``||g||^2``);
2. one ``all_to_all`` gathers the pieces of each matrix on its owner, which
   stacks equal shapes and runs the batched Newton-Schulz iteration;
3. the owner scales the result by ``lr * ||g|| / (||o|| + 1e-8)`` and a second
   ``all_to_all`` scatters the pieces back, where they are subtracted from the
   fp32 master shard.

So the reduce-scatter of the engine plus two bf16 all-to-alls carry all the
optimizer traffic, and every rank runs Newton-Schulz on ~1/world of the
matrices.

On one node (``comm="p2p"``, the default for CUDA ranks of one node; set
``LRB_DMUON_COMM=nccl`` for the collective path) the exchanges use no NCCL
call: the prologue writes each rank's pieces straight into its symmetric heap,
the rank raises a ready flag, and every rank pulls the pieces it needs from its
peers' heaps with P2P loads (``p2p_a2av_pull``) -- gradients to the owners'
Newton-Schulz stacks, scaled updates back.  The per-matrix ``||g||^2`` partials
and the "received a gradient" flags travel the same way (each rank pulls every
rank's small vector and reduces locally).  Reuse of a heap region across steps
needs no extra handshake: a rank rewrites its step-t gradient pieces only after
it pulled its step-t updates, which every owner published only after pulling
its step-t gradients, and symmetrically for the update region.  Under tensor parallelism (engine ``tp_group``) a TP-sharded matrix
is all-gathered over the TP group on its owner (the TP peers own the same
matrices), orthogonalised whole, and each peer keeps its slice, so the update
equals that of the unsharded matrix.  ``state_dict`` gathers the full per-parameter state in the layout
of ``torch.optim.Optimizer.state_dict`` with the reference's state keys
(``olympus/optim/muon_adamw_hybrid.py:118-170``).
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple, Type

import torch
import torch.distributed as dist

from llm_research_b200 import ops


@dataclass
class Segment:
    pid: int            # ParamInfo.index
    unit: int
    shard_off: int      # offset inside this rank's shard of the unit
    param_off: int      # offset inside the flattened parameter
    length: int


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def _is_hybrid(cls: type) -> bool:
    from olympus.optim.muon import Muon
    from olympus.optim.muon_adamw_hybrid import MuonAdamWHybrid

    return issubclass(cls, (MuonAdamWHybrid, Muon))


def _pure_muon(cls: type) -> bool:
    from olympus.optim.muon import Muon

    return issubclass(cls, Muon)


class ShardedHybridOptimizer:
    """Optimizer facade over the engine's shards (``step``/``zero_grad``/``state_dict``)."""

    def __init__(self, engine, optimizer_cls: Type[torch.optim.Optimizer], defaults: Dict[str, Any]) -> None:
        self.engine = engine
        self.optimizer_cls = optimizer_cls
        self.defaults = dict(defaults)
        self.param_groups: List[Dict[str, Any]] = [dict(self.defaults, params=[i.param for i in engine.params])]
        self.hybrid = _is_hybrid(optimizer_cls)
        self.state: Dict[Any, Any] = {}
        self.local_momentum: Dict[str, torch.Tensor] = {}
        world, rank = engine.world, engine.rank
        self.world, self.rank = world, rank
        dev = engine.device

        if not self.hybrid:
            # Elementwise optimizers run unchanged on flat shard parameters.
            self._flat = []
            for u in engine.units:
                p = torch.nn.Parameter(u.master, requires_grad=True)
                self._flat.append(p)
            self.inner = optimizer_cls(self._flat + [p for _, p in engine.local_params], **self.defaults)
            self.param_groups = self.inner.param_groups
            return

        pure = _pure_muon(optimizer_cls)
        max_ar = float(self.defaults.get("muon_max_aspect_ratio", 8.0))
        # Tensor-parallel shards (``_lrb_tp`` = concatenation dim): Muon acts on the full
        # matrix, gathered over the TP group on the owner (the TP peers own the same pids).
        tpg = getattr(engine, "tp_group", None)
        self.tp_world = dist.get_world_size(tpg) if tpg is not None else 1
        self.tp_dim = {i.index: getattr(i.param, "_lrb_tp", None) for i in engine.params} if tpg is not None else {}
        self.is_muon = {}
        for info in engine.params:
            shape = list(info.shape)
            if self.tp_dim.get(info.index) is not None:
                shape[self.tp_dim[info.index]] *= self.tp_world
            m = len(shape) == 2 and (pure or max(shape) <= min(shape) * max_ar)
            if pure and len(info.shape) != 2:
                raise ValueError(f"Muon only supports 2-D parameters, got {info.name} {info.shape}")
            self.is_muon[info.index] = m

        # ---- segments of this rank
        self.segments: List[Segment] = []
        for u in engine.units:
            lo, hi = rank * u.shard, (rank + 1) * u.shard
            for info in u.params:
                a, b = max(lo, info.offset), min(hi, info.offset + info.numel)
                if a < b:
                    self.segments.append(Segment(info.index, u.index, a - lo, a - info.offset, b - a))
        self.adam_segs = [s for s in self.segments if not self.is_muon[s.pid]]
        self.muon_segs = [s for s in self.segments if self.is_muon[s.pid]]

        # ---- per-unit state shards
        need_m = {s.unit for s in self.muon_segs}
        need_a = {s.unit for s in self.adam_segs}
        self.momentum = {ui: torch.zeros(engine.units[ui].shard, device=dev) for ui in need_m}
        self.exp_avg = {ui: torch.zeros(engine.units[ui].shard, device=dev) for ui in need_a}
        self.exp_avg_sq = {ui: torch.zeros(engine.units[ui].shard, device=dev) for ui in need_a}
        self.steps: Dict[int, int] = defaultdict(int)

        # ---- Muon ownership (global, deterministic)
        infos = {i.index: i for i in engine.params}
        muon_ids = sorted(i for i, m in self.is_muon.items() if m)
        self.muon_ids = muon_ids
        self.muon_pos = {pid: k for k, pid in enumerate(muon_ids)}
        loads = [0.0] * world
        self.owner: Dict[int, int] = {}
        for pid in sorted(muon_ids, key=lambda p: (-self._ns_cost(infos[p].shape), p)):
            r = min(range(world), key=lambda k: (loads[k], k))
            self.owner[pid] = r
            loads[r] += self._ns_cost(infos[pid].shape)
        self._build_exchange(infos)

    def _want_p2p(self) -> bool:
        import os

        eng = self.engine
        mode = os.environ.get("LRB_DMUON_COMM", "p2p").lower()
        if mode != "p2p" or self.world == 1 or eng.device.type != "cuda":
            return False
        from llm_research_b200.parallel.symm import single_node

        return single_node(eng.pg)

    @staticmethod
    def _ns_cost(shape: Tuple[int, ...]) -> float:
        m, n = shape
        s, l = min(m, n), max(m, n)
        return 4.0 * s * s * l + 2.0 * s ** 3

    def _pieces_of(self, info, r: int) -> Optional[Tuple[int, int]]:
        u = self.engine.units[info.unit]
        lo, hi = r * u.shard, (r + 1) * u.shard
        a, b = max(lo, info.offset), min(hi, info.offset + info.numel)
        return (a - info.offset, b - a) if a < b else None

    def _build_exchange(self, infos) -> None:
        eng, world, rank, dev = self.engine, self.world, self.rank, self.engine.device
        # send order: by (owner, pid); each Muon param has at most one segment per rank.
        seg_by_pid = {s.pid: s for s in self.muon_segs}
        self.send_order = sorted(self.muon_segs, key=lambda s: (self.owner[s.pid], s.pid))
        # every piece starts on a 16-byte boundary of the bf16 exchange buffers
        # (P2P pulls move 16-byte words); the padding is zero and never read back
        self.send_pos: Dict[int, int] = {}
        self.send_splits = [0] * world
        pos = 0
        for s in self.send_order:
            self.send_pos[s.pid] = pos
            pos += _pad8(s.length)
            self.send_splits[self.owner[s.pid]] += _pad8(s.length)
        self.send_total = pos
        # owned matrices, grouped by shape -> stack layout
        owned = [pid for pid in self.muon_ids if self.owner[pid] == rank]
        groups: Dict[Tuple[Tuple[int, int], Optional[int]], List[int]] = defaultdict(list)
        for pid in owned:
            groups[(infos[pid].shape, self.tp_dim.get(pid))].append(pid)
        self.groups = list(groups.items())
        self.stack_base: Dict[int, int] = {}
        base = 0
        for _, pids in self.groups:
            for pid in pids:
                self.stack_base[pid] = base
                base += infos[pid].numel
        self.stack_total = base
        # receive layout: for each source rank, pieces of owned matrices in pid order;
        # (recv offset, stack offset, length) segments map it onto the stack
        self.recv_splits = [0] * world
        self.r2s: List[Tuple[int, int, int]] = []
        pos = 0
        for r in range(world):
            for pid in owned:
                pc = self._pieces_of(infos[pid], r)
                if pc is None:
                    continue
                off, ln = pc
                self.r2s.append((pos, self.stack_base[pid] + off, ln))
                self.recv_splits[r] += _pad8(ln)
                pos += _pad8(ln)
        self.recv_total = pos
        self._bufs = None  # persistent exchange buffers and their segment views (first step)
        self.p2p = None
        if self._want_p2p():
            self.p2p = _P2PExchange(self)

    # ------------------------------------------------------------------ step
    def _views(self, ui: int, seg: Segment, buf: torch.Tensor) -> torch.Tensor:
        return buf[seg.shard_off: seg.shard_off + seg.length]

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        eng = self.engine
        eng.wait_grads()
        if not self.hybrid:
            for p, u in zip(self._flat, eng.units):
                p.grad = u.grad_shard
            self.inner.step()
            eng.refresh()
            return loss
        g = self.param_groups[0]
        pure = _pure_muon(self.optimizer_cls)
        lr_m = g["lr"] if pure else g["lr_muon"]
        wd_m = g.get("weight_decay", 0.0) if pure else g["weight_decay_muon"]
        mu = g["momentum"]
        ns_steps = g["ns_steps"]
        units = eng.units

        active = eng.touched_params(self.p2p.max_flags if self.p2p is not None else None)
        adam_segs = [s for s in self.adam_segs if s.pid in active]
        if adam_segs:
            for pid in sorted({s.pid for s in adam_segs}):
                self.steps[pid] += 1
            beta1, beta2 = g["betas"]
            ops.adamw_step(
                [units[s.unit].master[s.shard_off: s.shard_off + s.length] for s in adam_segs],
                [units[s.unit].grad_shard[s.shard_off: s.shard_off + s.length] for s in adam_segs],
                [self.exp_avg[s.unit][s.shard_off: s.shard_off + s.length] for s in adam_segs],
                [self.exp_avg_sq[s.unit][s.shard_off: s.shard_off + s.length] for s in adam_segs],
                [self.steps[s.pid] for s in adam_segs],
                lr=g["lr_adamw"], beta1=beta1, beta2=beta2, eps=g["eps"], weight_decay=g["weight_decay_adamw"],
            )

        # with the P2P exchange every rank takes part every step (lockstep epochs
        # keep the heap regions' reuse safe); a matrix without a gradient sends zeros
        if self.muon_ids and (self.p2p is not None or any(p in active for p in self.muon_ids)):
            self._muon_step(lr_m, mu, wd_m, ns_steps, active)
        self._step_local(lr_m, mu, wd_m, ns_steps)
        eng.refresh()
        return loss

    def _step_local(self, lr: float, mu: float, wd: float, ns_steps: int) -> None:
        """Muon on the engine's rank-local parameters (expert-parallel experts):
        every 2-D slice (one expert's matrix) gets its Nesterov direction, one
        batched Newton-Schulz per parameter orthogonalises all its experts at once."""
        for name, p in self.engine.local_params:
            if p.grad is None:
                continue
            mats = [p] if p.dim() == 2 else list(p.reshape(-1, p.shape[-2], p.shape[-1]).unbind(0))
            grads = [p.grad] if p.dim() == 2 else list(p.grad.reshape(-1, p.shape[-2], p.shape[-1]).unbind(0))
            buf = self.local_momentum.get(name)
            if buf is None:
                buf = self.local_momentum[name] = torch.zeros_like(p, dtype=torch.float32)
            bufs = [buf] if p.dim() == 2 else list(buf.reshape(-1, p.shape[-2], p.shape[-1]).unbind(0))
            outs, gnorm = ops.muon_prologue(mats, grads, bufs, lr, mu, wd)
            orth = ops.newton_schulz(torch.stack(outs), steps=ns_steps)
            ops.muon_epilogue(mats, list(orth.unbind(0)), gnorm, lr)

    def _exchange_buffers(self, xdt: torch.dtype):
        """send / recv / stack / back / upd buffers, allocated once, with the views that
        the segment copies between the receive layout and the stack use."""
        if self._bufs is None or self._bufs["dtype"] != xdt:
            dev = self.engine.device
            if self.p2p is not None:  # the two published regions live in the symmetric heap
                send, back = self.p2p.send, self.p2p.back
            else:
                send = torch.zeros(self.send_total, dtype=xdt, device=dev)
                back = torch.empty(self.recv_total, dtype=xdt, device=dev)
            recv = send if self.world == 1 else torch.empty(self.recv_total, dtype=xdt, device=dev)
            stack = torch.empty(self.stack_total, dtype=xdt, device=dev)
            upd = back if self.world == 1 else torch.empty(self.send_total, dtype=xdt, device=dev)
            self._bufs = dict(dtype=xdt, send=send, recv=recv, stack=stack, back=back, upd=upd,
                              recv_v=[recv[a: a + n] for a, _, n in self.r2s],
                              back_v=[back[a: a + n] for a, _, n in self.r2s],
                              stack_v=[stack[b: b + n] for _, b, n in self.r2s])
        return self._bufs

    @staticmethod
    def _copy_segments(dst, src) -> None:
        if dst:
            torch._foreach_copy_(dst, src)

    def _muon_step(self, lr: float, mu: float, wd: float, ns_steps: int, active) -> None:
        eng, units, dev = self.engine, self.engine.units, self.engine.device
        xdt = torch.bfloat16 if dev.type == "cuda" else torch.float32  # exchange / Newton-Schulz dtype
        B = self._exchange_buffers(xdt)
        send, recv, stack, back, upd = B["send"], B["recv"], B["stack"], B["back"], B["upd"]
        send.zero_()  # matrices without a gradient keep u = 0 -> zero update, no decay
        outs, segs = [], []
        for s in self.send_order:
            if s.pid in active:
                pos = self.send_pos[s.pid]
                outs.append(send[pos: pos + s.length])
                segs.append(s)
        gnorm_seg = ops.muon_prologue_into(
            [units[s.unit].master[s.shard_off: s.shard_off + s.length] for s in segs],
            [units[s.unit].grad_shard[s.shard_off: s.shard_off + s.length] for s in segs],
            [self.momentum[s.unit][s.shard_off: s.shard_off + s.length] for s in segs],
            outs, float(lr), float(mu), float(wd),
        )
        # per-matrix ||g||^2 summed over the ranks holding its pieces
        gsq = torch.zeros(len(self.muon_ids), device=dev)
        idx = torch.tensor([self.muon_pos[s.pid] for s in segs], device=dev, dtype=torch.long)
        if segs:
            gsq.index_add_(0, idx, gnorm_seg.pow(2))
        if self.p2p is not None:
            gsq = self.p2p.exchange_grads(gsq, recv)  # pieces to the owners + sum of the norm partials
        elif self.world > 1:
            dist.all_reduce(gsq, group=eng.pg)
        if self.tp_world > 1:  # ||g||^2 of a TP-sharded matrix: sum over its shards
            mask = torch.tensor([self.tp_dim.get(p) is not None for p in self.muon_ids], device=dev)
            part = gsq * mask
            dist.all_reduce(part, group=eng.tp_group)
            gsq = torch.where(mask, part, gsq)
        if self.world > 1 and self.p2p is None:
            dist.all_to_all_single(recv, send, self.recv_splits, self.send_splits, group=eng.pg)
        self._copy_segments(B["stack_v"], B["recv_v"])
        gnorm = gsq.sqrt()
        base = 0
        for (shape, tpd), pids in self.groups:
            n = len(pids)
            numel = shape[0] * shape[1]
            block = stack[base: base + n * numel].view(n, shape[0], shape[1])
            if tpd is None:
                o = ops.newton_schulz(block, steps=ns_steps)
                onorm = torch.linalg.vector_norm(o.flatten(1), dim=1, dtype=torch.float32)
            else:
                parts = [torch.empty_like(block) for _ in range(self.tp_world)]
                dist.all_gather(parts, block.contiguous(), group=eng.tp_group)
                o_full = ops.newton_schulz(torch.cat(parts, dim=1 + tpd), steps=ns_steps)
                onorm = torch.linalg.vector_norm(o_full.flatten(1), dim=1, dtype=torch.float32)
                o = o_full.chunk(self.tp_world, dim=1 + tpd)[dist.get_rank(eng.tp_group)]
            gn = gnorm[torch.tensor([self.muon_pos[p] for p in pids], device=dev)]
            scale = (lr * gn / (onorm + 1e-8)).view(n, 1, 1)
            torch.mul(o, scale, out=block)  # fp32 product, one rounding into the stack
            base += n * numel
        self._copy_segments(B["back_v"], B["stack_v"])
        if self.p2p is not None:
            self.p2p.exchange_updates(upd)
        elif self.world > 1:
            dist.all_to_all_single(upd, back, self.send_splits, self.recv_splits, group=eng.pg)
        masters, deltas = [], []
        for s in self.send_order:
            if s.pid in active:
                pos = self.send_pos[s.pid]
                masters.append(units[s.unit].master[s.shard_off: s.shard_off + s.length])
                deltas.append(upd[pos: pos + s.length])
        ops.axpy_list(masters, deltas, -1.0)

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.engine.zero_grad()

    # ---------------------------------------------------------- checkpoints
    @torch.no_grad()
    def state_dict(self) -> Dict[str, Any]:
        eng = self.engine
        groups = [{k: v for k, v in self.param_groups[0].items() if k != "params"}]
        groups[0]["params"] = [i.index for i in eng.params]
        if not self.hybrid:
            return {"state": {}, "param_groups": groups, "inner": self.inner.state_dict()}
        state: Dict[int, Dict[str, Any]] = {}
        full = {}
        for name, bufs in (("momentum_buffer", self.momentum), ("exp_avg", self.exp_avg), ("exp_avg_sq", self.exp_avg_sq)):
            for u in eng.units:
                src = bufs.get(u.index)
                if src is None:
                    src = torch.zeros(u.shard, device=eng.device)
                full[(name, u.index)] = eng.full_flat(u, src)
        for info in eng.params:
            sl = slice(info.offset, info.offset + info.numel)
            if self.is_muon[info.index]:
                state[info.index] = {
                    "type": "muon",
                    "momentum_buffer": full[("momentum_buffer", info.unit)][sl].view(info.shape).cpu().clone(),
                }
            else:
                state[info.index] = {
                    "type": "adamw",
                    "step": int(self._global_step(info.index)),
                    "exp_avg": full[("exp_avg", info.unit)][sl].view(info.shape).cpu().clone(),
                    "exp_avg_sq": full[("exp_avg_sq", info.unit)][sl].view(info.shape).cpu().clone(),
                }
        return {"state": state, "param_groups": groups}

    def steps_taken(self, pid: int) -> int:
        return self.steps.get(pid, 0)

    def _global_step(self, pid: int) -> int:
        t = torch.tensor([self.steps.get(pid, 0)], dtype=torch.long, device=self.engine.device)
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.engine.pg)
        return int(t.item())

    @torch.no_grad()
    def load_state_dict(self, sd: Dict[str, Any]) -> None:
        eng = self.engine
        if sd.get("param_groups"):
            for k, v in sd["param_groups"][0].items():
                if k != "params":
                    self.param_groups[0][k] = v
        if not self.hybrid:
            if "inner" in sd:
                self.inner.load_state_dict(sd["inner"])
            return
        st = sd.get("state", {})
        for info in eng.params:
            ent = st.get(info.index) or st.get(str(info.index))
            if ent is None:
                continue
            u = eng.units[info.unit]
            lo = eng.rank * u.shard
            a, b = max(lo, info.offset), min(lo + u.shard, info.offset + info.numel)
            if a >= b:
                if ent.get("type") == "adamw":
                    self.steps[info.index] = int(ent.get("step", 0))
                continue
            src_sl = slice(a - info.offset, b - info.offset)
            dst_sl = slice(a - lo, b - lo)
            if ent.get("type") == "muon" and info.unit in self.momentum:
                self.momentum[info.unit][dst_sl].copy_(ent["momentum_buffer"].reshape(-1)[src_sl])
            elif ent.get("type") == "adamw" and info.unit in self.exp_avg:
                self.exp_avg[info.unit][dst_sl].copy_(ent["exp_avg"].reshape(-1)[src_sl])
                self.exp_avg_sq[info.unit][dst_sl].copy_(ent["exp_avg_sq"].reshape(-1)[src_sl])
                self.steps[info.index] = int(ent.get("step", 0))


class _P2PExchange:
    """The optimizer's exchanges over a symmetric heap of the engine's group.

    Heap layout (same offsets on every rank): the gradient-piece region (the
    largest send layout of any rank), the update region (the largest receive
    layout), one small fp32 vector slot per kind (norm partials, gradient
    flags), and one ready flag per kind.  Each exchange: the rank's data is in
    its own region, it raises its flag to the exchange's epoch, and it pulls
    its pieces from every rank's region once that rank's flag reached the
    epoch."""

    FLAG_GRADS, FLAG_UPDATES, FLAG_TOUCHED = 0, 1, 2

    def __init__(self, opt: "ShardedHybridOptimizer") -> None:
        from llm_research_b200.parallel.symm import SymmetricHeap

        eng = opt.engine
        self.opt, self.world, self.rank, dev = opt, opt.world, opt.rank, eng.device
        splits: List[Any] = [None] * self.world
        dist.all_gather_object(splits, list(opt.send_splits), group=eng.pg)
        self.all_send = [list(map(int, x)) for x in splits]  # all_send[r][o]: r's elements for owner o
        max_send = max(sum(x) for x in self.all_send)
        max_recv = max(sum(self.all_send[r][o] for r in range(self.world)) for o in range(self.world))
        self.n_small = max(len(opt.muon_ids), len(eng.params), 1)
        small = _pad8(self.n_small) * 4
        need = 2 * max_send + 2 * max_recv + 2 * small + 4096
        self.heap = heap = SymmetricHeap(need, group=eng.pg, device=dev)
        self.send_off = heap.alloc(2 * max(max_send, 8))
        self.back_off = heap.alloc(2 * max(max_recv, 8))
        self.small_off = [heap.alloc(small), heap.alloc(small)]  # norm partials, gradient flags
        self.flag_off = [heap.alloc(4) for _ in range(3)]
        self.send = heap.view(self.send_off, (opt.send_total,), torch.bfloat16)
        self.back = heap.view(self.back_off, (opt.recv_total,), torch.bfloat16)
        self.small = [heap.view(o, (self.n_small,), torch.float32) for o in self.small_off]
        self.flags = [heap.view(o, (1,), torch.int32) for o in self.flag_off]
        self.epoch = [0, 0, 0]
        W, me, A = self.world, self.rank, self.all_send

        def prefix(xs, k):
            return sum(xs[:k])

        # gradients: from rank r, r's block for owner `me`, into my receive layout
        self.plan_grads = self._plan(
            [self.send_off + 2 * prefix(A[r], me) for r in range(W)],
            [2 * prefix([A[q][me] for q in range(W)], r) for r in range(W)],
            [2 * A[r][me] for r in range(W)], dev)
        # updates: from owner r, its back-region block for source `me`, into my send layout
        self.plan_updates = self._plan(
            [self.back_off + 2 * prefix([A[q][r] for q in range(W)], me) for r in range(W)],
            [2 * prefix(A[me], r) for r in range(W)],
            [2 * A[me][r] for r in range(W)], dev)
        self.gather_small = torch.empty(W, _pad8(self.n_small), dtype=torch.float32, device=dev)

    @staticmethod
    def _plan(src, dst, lens, dev) -> torch.Tensor:
        return torch.tensor([src, dst, lens], dtype=torch.int64, device=dev)

    def _publish_and_pull(self, kind: int, dst: torch.Tensor, plan: torch.Tensor) -> None:
        from llm_research_b200._ext import native

        self.epoch[kind] += 1
        C = native()
        C.ep_flag_set(self.flags[kind], self.epoch[kind])
        C.p2p_a2av_pull(dst, self.heap.bases, plan, self.flag_off[kind], self.world, self.epoch[kind], self.heap.err)

    def _small_plan(self, slot: int, n: int) -> torch.Tensor:
        row = _pad8(self.n_small) * 4
        return self._plan([self.small_off[slot]] * self.world, [r * row for r in range(self.world)],
                          [_pad8(n) * 4] * self.world, self.gather_small.device)

    def exchange_grads(self, gsq: torch.Tensor, recv: torch.Tensor) -> torch.Tensor:
        """Publishes the gradient pieces (already in the heap) and the norm partials;
        pulls this rank's pieces into ``recv``; returns the summed partials."""
        n = gsq.numel()
        self.small[0][:n].copy_(gsq)
        if not hasattr(self, "_plan_gsq"):
            self._plan_gsq = self._small_plan(0, n)
        self._publish_and_pull(self.FLAG_GRADS, recv, self.plan_grads)
        from llm_research_b200._ext import native

        # same flag and epoch: the partials were written before it was raised
        native().p2p_a2av_pull(self.gather_small, self.heap.bases, self._plan_gsq, self.flag_off[self.FLAG_GRADS],
                               self.world, self.epoch[self.FLAG_GRADS], self.heap.err)
        return self.gather_small[:, :n].sum(0)

    def exchange_updates(self, upd: torch.Tensor) -> None:
        self._publish_and_pull(self.FLAG_UPDATES, upd, self.plan_updates)

    def max_flags(self, flags: torch.Tensor) -> torch.Tensor:
        n = flags.numel()
        self.small[1][:n].copy_(flags)
        if not hasattr(self, "_plan_flags"):
            self._plan_flags = self._small_plan(1, n)
        self._publish_and_pull(self.FLAG_TOUCHED, self.gather_small, self._plan_flags)
        return self.gather_small[:, :n].amax(0)

    def close(self) -> None:
        self.heap.close()
