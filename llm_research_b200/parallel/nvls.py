"""Multicast symmetric memory for NVSwitch (NVLS) collectives on one node.

A :class:`MulticastHeap` is one allocation of the same size on every rank of a
group, made with torch's symmetric-memory allocator
(``torch.distributed._symmetric_memory``, CUDA backend) and bound to an NVLink
multicast object.  Every byte of it has three kinds of address:

* this rank's unicast address (a normal device pointer; :meth:`view` returns a
  tensor over it);
* each peer's unicast address (``bases``, an int64 device table: plain P2P loads
  and stores over NVLink, used for the epoch flags);
* one multicast address (:meth:`mc`) that names the copies of all ranks at once:
  ``multimem.ld_reduce`` through it returns the sum over the ranks, computed in
  the switch, and ``multimem.st`` writes every rank's copy.

The kernels that use it are in ``csrc/comm/nvls.cu`` (all-reduce, the FSDP
reduce-scatter, the once-per-step parameter broadcast and DiLoCo's outer step).
torch only provides the allocation, the multicast binding and the handle
exchange; no torch or NCCL collective runs on this path.

Multicast needs NVSwitch and driver support; :class:`NVLSUnavailable` is raised
when the allocation comes back without a multicast address.  A rank that dies
while its memory is bound to the multicast object can fault the other GPUs, so
the failure-detection tests never use this path.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.distributed as dist

from llm_research_b200._ext import native

_ERR_NAMES = {41: "NVLS: timed out waiting for a peer's ready flag",
              42: "NVLS: timed out waiting for the peers' results",
              43: "NVLS: timed out waiting for a peer to release a buffer"}


class NVLSUnavailable(RuntimeError):
    """The group's memory could not be bound to a multicast object."""


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class MulticastHeap:
    def __init__(self, nbytes: int, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None) -> None:
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = _round_up(max(int(nbytes), 1 << 16), 1 << 21)
        try:
            symm_mem.set_backend("CUDA")
        except Exception:  # already chosen by an earlier allocation
            pass
        self.buf = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=self.device)
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        if mc == 0:
            raise NVLSUnavailable("symmetric memory came back without a multicast address "
                                  "(no NVSwitch multicast on this node)")
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        # The tensor may start at an offset inside the allocation that the
        # unicast and multicast base addresses refer to.
        self._off = int(self.buf.data_ptr()) - ptrs[self.rank]
        self.mc_base = mc + self._off
        self.peer_bases = [p + self._off for p in ptrs]
        self.bases = torch.tensor(self.peer_bases, dtype=torch.int64, device=self.device)
        self.err = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._host_err = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        self.buf.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every copy is zeroed before anyone signals
        self._next = 0
        self._closed = False

    # ------------------------------------------------------------- carving
    def alloc(self, nbytes: int, align: int = 256) -> int:
        """Offset of a new zero-initialised sub-buffer (same on every rank)."""
        off = _round_up(self._next, align)
        if off + nbytes > self.nbytes:
            raise MemoryError(f"multicast heap exhausted: need {off + nbytes} of {self.nbytes} bytes")
        self._next = off + nbytes
        return off

    def view(self, offset: int, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        """This rank's tensor view of a sub-buffer."""
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return self.buf[offset: offset + nbytes].view(dtype).view(tuple(shape))

    def mc(self, offset: int) -> int:
        """Multicast address of byte ``offset``."""
        return self.mc_base + int(offset)

    # -------------------------------------------------------------- errors
    def poll_error(self) -> None:
        """Raise if an earlier kernel recorded a failed wait (reads the last
        call's copy of the error word; no sync)."""
        code = int(self._host_err[0])
        if code:
            raise RuntimeError(f"NVLS collective failed on rank {self.rank}: {_ERR_NAMES.get(code, f'error {code}')}")
        self._host_err.copy_(self.err, non_blocking=True)

    def check(self) -> None:
        torch.cuda.synchronize(self.device)
        self._host_err.copy_(self.err)
        self.poll_error()

    # ------------------------------------------------------------- teardown
    def close(self) -> None:
        """Collective: no rank drops the allocation while a peer may still use it."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.handle = None
        self.buf = None
        self._closed = True


class NVLSAllReduce:
    """In-place sum (times ``scale``) over a group of a tensor that lives in a
    :class:`MulticastHeap` -- used for DiLoCo's pseudo-gradients and available
    for any replicated-gradient all-reduce.  Each rank reduces one 1/world slice
    in the switch and multicasts the result."""

    def __init__(self, numel: int, dtype: torch.dtype = torch.float32, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None, heap: Optional[MulticastHeap] = None) -> None:
        esize = torch.empty((), dtype=dtype).element_size()
        nbytes = _round_up(numel * esize, 16)
        self.heap = heap or MulticastHeap(nbytes + 4096, group=group, device=device)
        self.world, self.rank = self.heap.world, self.heap.rank
        self.data_off = self.heap.alloc(nbytes)
        self.flag_off = self.heap.alloc(8 * self.world)
        self.numel = numel
        self.buffer = self.heap.view(self.data_off, (nbytes // esize,), dtype)
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.heap.device)
        self.epoch = 0

    def tensor(self) -> torch.Tensor:
        """The ``numel`` elements to fill before :meth:`run` (result in place)."""
        return self.buffer[: self.numel]

    def run(self, scale: float = 1.0) -> torch.Tensor:
        self.epoch += 1
        native().nvls_all_reduce(self.buffer, self.heap.mc(self.data_off), self.heap.bases, self.flag_off,
                                 self.rank, self.world, self.epoch, float(scale), self.counter, self.heap.err)
        return self.tensor()
