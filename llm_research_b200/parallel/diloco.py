"""DiLoCo: islands that train locally and synchronise every ``inner_steps``.

Topology (:func:`make_diloco_groups`): ``world = R × S`` ranks form ``R``
replicas ("islands") of ``S`` ranks; inside an island the model is sharded
with :class:`~llm_research_b200.parallel.fsdp.FlatShardEngine` over the
island group, and rank ``i·S + p`` of every island holds the same shard
positions, so the outer synchronisation is shard-wise over the *replica
group* ``{p, S + p, 2S + p, ...}``.

Outer step (Nesterov, the DiLoCo recipe of Douillard et al. 2023, settings
of ``configs/distributed/diloco.yaml:1-11`` in the reference: 500 inner steps,
outer lr 0.7, outer momentum 0.9):

    delta  = anchor - local                 (pseudo-gradient, fp32)
    delta  = mean over live replicas
    m      = mu * m + delta
    anchor = anchor - lr * (delta + mu * m)
    local  = anchor

Transports:

* ``p2p`` (one node, fixed membership): three kernels of ``_C`` on symmetric
  memory -- ``diloco_push`` computes the pseudo-gradient and stores each
  owner's slice into its receive slot, ``diloco_reduce_nesterov`` averages the
  slots and applies the momentum / anchor update to the owned slice (fused),
  and ``p2p_pull`` gathers the updated anchor slices;
* ``collective`` -- ``all_reduce`` over the replica group (NCCL or gloo), or,
  with ``quantize_bits=4``, an all-gather of int4-absmax-compressed
  pseudo-gradients (1/8 of the fp32 bytes) averaged after dequantisation.

Fault tolerance (host side, no GPU fault needed): a heartbeat monitor marks
replicas whose heartbeat is older than its timeout as dead; at every outer
step the lowest live rank of a replica group publishes the roster (live ranks
plus ranks that asked to join) in the store, every listed rank builds a
:class:`~llm_research_b200.parallel.fault.RosterGroup` for it (the dead rank
is not needed) and a joining rank receives anchor and momentum by broadcast.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from llm_research_b200.parallel.fault import HeartbeatMonitor, RosterGroup, default_store
from llm_research_b200.utils.nvtx import nvtx_fn


@dataclass
class DiLoCoConfig:
    inner_steps: int = 500
    outer_lr: float = 0.7
    outer_momentum: float = 0.9
    nesterov: bool = True
    quantize_bits: int = 0          # 0: exact fp32 exchange; 4: int4 absmax (group 128) pseudo-gradients
    fault_tolerance: bool = True
    max_island_failures: int = 2
    comm: str = "auto"              # auto | p2p | nvls | collective


def make_diloco_groups(num_replicas: int) -> Tuple[Optional[dist.ProcessGroup], dist.ProcessGroup, List[int], int]:
    """``(island_group, replica_group, replica_ranks, island_index)`` for this rank.
    Every rank creates every group, in the same order."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if world % num_replicas:
        raise ValueError(f"world size {world} is not a multiple of {num_replicas} replicas")
    S = world // num_replicas
    island_group = None
    for i in range(num_replicas):
        g = dist.new_group(list(range(i * S, (i + 1) * S)))
        if i == rank // S:
            island_group = g
    replica_group, replica_ranks = None, []
    for p in range(S):
        ranks = [p + i * S for i in range(num_replicas)]
        g = dist.new_group(ranks)
        if p == rank % S:
            replica_group, replica_ranks = g, ranks
    return island_group, replica_group, replica_ranks, rank // S


class DiLoCo:
    def __init__(self, shards: Sequence[torch.Tensor], replica_group: dist.ProcessGroup, replica_ranks: Sequence[int],
                 config: Optional[DiLoCoConfig] = None, monitor: Optional[HeartbeatMonitor] = None,
                 on_update=None, tag: str = "diloco") -> None:
        """``shards``: this rank's fp32 master tensors (updated in place at every
        outer step); ``on_update``: called after they change (e.g. ``engine.refresh``)."""
        self.cfg = config or DiLoCoConfig()
        self.shards = list(shards)
        self.group = replica_group
        self.members = list(replica_ranks)
        self.initial = list(replica_ranks)
        self.rank = dist.get_rank()
        self.monitor = monitor
        self.on_update = on_update
        self.tag = tag
        self.device = self.shards[0].device
        self.numel = sum(s.numel() for s in self.shards)
        R = len(self.members)
        self.padded = -(-self.numel // (4 * R * 8)) * (4 * R * 8)
        self.local = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        self._flatten()
        self.anchor = self.local.clone()
        self.momentum: Optional[torch.Tensor] = None
        self.inner_step = 0
        self.outer_steps = 0
        self._epoch = 0
        self.heap = None
        comm = self.cfg.comm
        if comm == "auto":
            comm = "p2p" if self._p2p_possible() else "collective"
        self.comm = comm
        if self.comm == "nvls":
            from llm_research_b200.parallel.nvls import NVLSUnavailable
            from llm_research_b200.parallel.symm import single_node

            try:
                if not (self.device.type == "cuda" and len(self.members) > 1 and self.cfg.quantize_bits == 0
                        and isinstance(self.group, dist.ProcessGroup) and single_node(self.group)):
                    raise NVLSUnavailable("the replica group is not a single-node process group")
                # A replica that dies while its memory is bound to a multicast
                # object can fault its peers' GPUs: with replica drop / rejoin
                # enabled (a heartbeat monitor), the plain P2P path is used.
                if self.cfg.fault_tolerance and self.monitor is not None:
                    raise NVLSUnavailable("replica drop / rejoin is enabled")
                self._setup_nvls()
            except NVLSUnavailable:
                self.comm = "p2p" if self._p2p_possible() else "collective"
        if self.comm == "p2p":
            self._setup_p2p()
        elif self.comm != "nvls":
            self.momentum = torch.zeros(self.padded, dtype=torch.float32, device=self.device)

    # ------------------------------------------------------------- plumbing
    def _p2p_possible(self) -> bool:
        from llm_research_b200.parallel.symm import single_node

        # The fused P2P kernel implements the Nesterov form only; heavy-ball
        # momentum (nesterov=False) takes the NVLS or collective path.
        return (self.device.type == "cuda" and len(self.members) > 1 and self.cfg.quantize_bits == 0
                and self.cfg.nesterov and single_node(self.group))

    def _setup_p2p(self) -> None:
        from llm_research_b200.parallel.symm import SymmetricHeap

        R = len(self.members)
        shard = self.padded // R
        self.heap = heap = SymmetricHeap(R * shard * 4 + shard * 4 + 4096, group=self.group, device=self.device)
        self.recv_off = heap.alloc(R * shard * 4)
        self.ready_off = heap.alloc(4 * R)
        self.consumed_off = heap.alloc(4)
        self.out_off = heap.alloc(shard * 4)
        self.outready_off = heap.alloc(4)
        self.recv = heap.view(self.recv_off, (R * shard,), torch.float32)
        self.ready = heap.view(self.ready_off, (R,), torch.int32)
        self.consumed = heap.view(self.consumed_off, (1,), torch.int32)
        self.out = heap.view(self.out_off, (shard,), torch.float32)
        self.outready = heap.view(self.outready_off, (1,), torch.int32)
        self.counters = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.my = self.members.index(self.rank)
        self.momentum = torch.zeros(shard, dtype=torch.float32, device=self.device)

    def _setup_nvls(self) -> None:
        from llm_research_b200.parallel.nvls import NVLSAllReduce

        R = len(self.members)
        self.nvls = NVLSAllReduce(self.padded, dtype=torch.float32, group=self.group, device=self.device)
        self.my = self.members.index(self.rank)
        per = -(-(self.padded // 4) // R)  # 16-byte vectors in this rank's slice
        self.momentum = torch.zeros(per * 4, dtype=torch.float32, device=self.device)
        self.heap = self.nvls.heap

    def _flatten(self) -> None:
        o = 0
        for s in self.shards:
            self.local[o: o + s.numel()].copy_(s.reshape(-1))
            o += s.numel()

    def _unflatten(self, src: torch.Tensor) -> None:
        o = 0
        for s in self.shards:
            s.copy_(src[o: o + s.numel()].view_as(s))
            o += s.numel()
        if self.on_update is not None:
            self.on_update()

    # ---------------------------------------------------------------- public
    def step(self) -> bool:
        """Call after every inner optimizer step; runs the outer step every ``inner_steps``."""
        self.inner_step += 1
        if self.inner_step % self.cfg.inner_steps == 0:
            self.outer_step()
            return True
        return False

    @torch.no_grad()
    @nvtx_fn("lrb/diloco/outer")
    def outer_step(self, _roster: Optional[Tuple[List[int], List[int]]] = None) -> None:
        self._flatten()
        joiners: List[int] = []
        if _roster is not None:
            joiners = self._adopt(*_roster)
        elif self.cfg.fault_tolerance and self.monitor is not None:
            joiners = self._update_roster()
        self._epoch += 1
        if self.comm == "nvls" and self.members == self.initial and not joiners:
            self._outer_nvls()
        elif self.comm == "p2p" and self.members == self.initial and not joiners:
            self._outer_p2p()
        else:
            self._outer_collective(len(self.members) - len(joiners))
        self.outer_steps += 1
        self._unflatten(self.anchor)

    # ------------------------------------------------------------ transports
    def _outer_p2p(self) -> None:
        from llm_research_b200._ext import native

        C = native()
        R = len(self.members)
        shard = self.padded // R
        C.diloco_push(self.anchor, self.local, self.heap.bases, self.recv_off, self.ready_off, self.consumed_off,
                      self.my, R, self._epoch, self.counters[0:1], self.heap.err)
        mine = self.anchor[self.my * shard: (self.my + 1) * shard]
        C.diloco_reduce_nesterov(self.recv, mine, self.momentum, self.out, R, self.cfg.outer_lr,
                                 self.cfg.outer_momentum if self.cfg.nesterov else 0.0, self.ready, self.consumed,
                                 self.outready, self._epoch, self.counters[1:2], self.heap.err)
        C.p2p_pull(self.anchor, self.heap.bases, self.out_off, self.outready_off, R, self._epoch, self.heap.err)
        self.heap.poll_error()

    def _outer_nvls(self) -> None:
        """Pseudo-gradients summed in the switch, the momentum step on this rank's
        slice and the new anchor multicast back: one kernel (``nvls_diloco_outer``)."""
        from llm_research_b200._ext import native

        ar = self.nvls
        buf = ar.tensor()
        torch.sub(self.anchor, self.local, out=buf)
        ar.epoch += 1
        native().nvls_diloco_outer(ar.buffer, ar.heap.mc(ar.data_off), ar.heap.bases, ar.flag_off, self.anchor,
                                   self.momentum, ar.rank, ar.world, ar.epoch, self.cfg.outer_lr,
                                   self.cfg.outer_momentum, self.cfg.nesterov, ar.counter, ar.heap.err)
        self.anchor.copy_(buf)
        ar.heap.poll_error()

    def _outer_collective(self, contributors: int) -> None:
        R = len(self.members)
        delta = self.anchor - self.local  # zero on a rank that just joined
        if self.cfg.quantize_bits == 4 and R > 1:
            delta = self._mean_int4(delta, contributors)
        elif R > 1:
            self._all_reduce(delta)
            delta.div_(contributors)
        if self.momentum is None or self.momentum.numel() != self.padded:
            self.momentum = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        mu = self.cfg.outer_momentum
        self.momentum.mul_(mu).add_(delta)
        if self.cfg.nesterov:
            self.anchor.sub_(self.cfg.outer_lr * (delta + mu * self.momentum))
        else:
            self.anchor.sub_(self.cfg.outer_lr * self.momentum)

    def _all_reduce(self, t: torch.Tensor) -> None:
        if isinstance(self.group, RosterGroup):
            self.group.all_reduce(t)
        else:
            dist.all_reduce(t, group=self.group)

    def _broadcast(self, t: torch.Tensor, src: int) -> None:
        if isinstance(self.group, RosterGroup):
            self.group.broadcast(t, src)
        else:
            dist.broadcast(t, src=src, group=self.group)

    def _all_gather(self, outs, t: torch.Tensor) -> None:
        if isinstance(self.group, RosterGroup):
            self.group.all_gather(outs, t)
        else:
            dist.all_gather(outs, t, group=self.group)

    def _mean_int4(self, delta: torch.Tensor, contributors: int) -> torch.Tensor:
        from llm_research_b200 import ops

        R = len(self.members)
        q, scale = ops.int4_quantize(delta.view(-1, 128), 128)
        qs = [torch.empty_like(q) for _ in range(R)]
        ss = [torch.empty_like(scale) for _ in range(R)]
        self._all_gather(qs, q)
        self._all_gather(ss, scale)
        out = torch.zeros_like(delta)
        for qi, si in zip(qs, ss):
            out += ops.int4_dequantize(qi, si, 128).reshape(-1)
        return out.div_(contributors)

    # ----------------------------------------------------------- membership
    # Store keys (per replica group g = first rank of the initial group):
    #   <tag>/roster/<g>/<epoch> = "m0,m1,...|j0,..."  members | joiners of that outer step
    #   <tag>/join/<g>/<rank>    = "1"                 rank asks to (re)join
    def _roster_key(self, epoch: int) -> str:
        return f"{self.tag}/roster/{self.initial[0]}/{epoch}"

    def _join_key(self, rank: int) -> str:
        return f"{self.tag}/join/{self.initial[0]}/{rank}"

    def _update_roster(self) -> List[int]:
        store = default_store()
        alive = set(self.monitor.live_ranks()) | {self.rank}
        live = [r for r in self.members if r in alive]
        key = self._roster_key(self._epoch + 1)
        if self.rank == min(live):
            joiners = []
            for r in self.initial:
                if r not in live and store.check([self._join_key(r)]):
                    joiners.append(r)
                    store.delete_key(self._join_key(r))
            store.set(key, ",".join(map(str, live)) + "|" + ",".join(map(str, joiners)))
        else:
            store.wait([key])
        m, j = store.get(key).decode().split("|")
        members = [int(x) for x in m.split(",") if x]
        joiners = [int(x) for x in j.split(",") if x]
        lost = len(self.initial) - len(members)
        if lost > self.cfg.max_island_failures:
            raise RuntimeError(f"{lost} replicas lost, more than max_island_failures={self.cfg.max_island_failures}")
        return self._adopt(members, joiners)

    def _adopt(self, members: List[int], joiners: List[int]) -> List[int]:
        roster = sorted(set(members) | set(joiners))
        if roster != self.members or joiners:
            self.members = roster
            self.group = RosterGroup(roster, f"{self.tag}/{self.initial[0]}/{self._epoch + 1}", self.device)
        if joiners:
            src = min(members)
            if self.momentum is None or self.momentum.numel() != self.padded:
                self.momentum = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
            self._broadcast(self.anchor, src)
            self._broadcast(self.momentum, src)
            if self.rank in joiners:
                self.local.copy_(self.anchor)
        return joiners

    def rejoin(self, timeout_s: float = 300.0) -> None:
        """(Re)join the replica group: announce, wait for the first outer step
        whose roster lists this rank, receive anchor and momentum, take part."""
        import time

        store = default_store()
        store.set(self._join_key(self.rank), "1")
        if self.monitor is not None:
            self.monitor._paused.clear()
            self.monitor.beat()
        e = self._epoch
        deadline = time.time() + timeout_s
        while True:
            key = self._roster_key(e + 1)
            store.wait([key])
            m, j = store.get(key).decode().split("|")
            joiners = [int(x) for x in j.split(",") if x]
            if self.rank in joiners:
                break
            e += 1
            if time.time() > deadline:
                raise TimeoutError("no outer step admitted this rank")
        self._epoch = e
        self.outer_step(_roster=([int(x) for x in m.split(",") if x], joiners))

    def close(self) -> None:
        if self.heap is not None:
            self.heap.close()
            self.heap = None
