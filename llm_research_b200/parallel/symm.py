"""Symmetric device memory over CUDA IPC for the ranks of one node.

Every rank allocates one device heap of the same size (``cudaMalloc``),
exports it with a CUDA IPC handle and opens the heaps of its peers, so a
kernel of ``llm_research_b200._C`` can load from and store to another GPU's
heap over NVLink with plain loads and stores.  Sub-buffers are carved out
with :meth:`SymmetricHeap.alloc` in the same order on every rank, so a buffer
has the same offset in every heap; kernels get the table of heap base
addresses (``bases``, int64 on the device) and the offset.

No multicast object is created and NVLS is not used: peer access is plain
P2P.  The process group is used once, to exchange the 64-byte handles.

Teardown (:meth:`close`) is collective: every rank closes its peer mappings
after a barrier, and frees its own heap after a second barrier.
"""

from __future__ import annotations

import os
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from llm_research_b200._ext import native

_ERR_NAMES = {11: "timed out waiting for a peer's data flag", 12: "timed out waiting for a peer to free its slot",
              21: "tensor parallel: timed out waiting for a peer", 22: "tensor parallel: timed out waiting for "
              "a slot", 23: "tensor parallel: timed out waiting for a gathered chunk",
              31: "expert parallel: timed out waiting for an owner's output", 32: "expert parallel: timed out "
              "waiting for an owner to release its slots", 33: "expert parallel: routing index outside the "
              "buffers (row skipped)"}


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def single_node(group: Optional[dist.ProcessGroup] = None) -> bool:
    """True when every rank of ``group`` runs on this node (IPC-reachable)."""
    world = dist.get_world_size(group)
    local = int(os.environ.get("LOCAL_WORLD_SIZE", world))
    return local >= world


class SymmetricHeap:
    def __init__(self, nbytes: int, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None) -> None:
        C = native()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.nbytes = _round_up(max(int(nbytes), 1 << 16), 1 << 21)
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._dev = dev
        self.base, handle = C.symm_alloc(self.nbytes, dev)
        handles: List[Optional[bytes]] = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=group)
        self._opened: List[int] = []
        bases: List[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self.base)
            else:
                p = C.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), dev)
                self._opened.append(p)
                bases.append(p)
        self.peer_bases = bases
        self.bases = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.err = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._host_err = torch.zeros(4, dtype=torch.int32, pin_memory=True)
        self._next = 0
        self._closed = False

    # ------------------------------------------------------------- carving
    def alloc(self, nbytes: int, align: int = 256) -> int:
        """Offset of a new zero-initialised sub-buffer (same on every rank)."""
        off = _round_up(self._next, align)
        if off + nbytes > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted: need {off + nbytes} of {self.nbytes} bytes")
        self._next = off + nbytes
        return off

    def view(self, offset: int, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        """Local tensor view of a sub-buffer (no ownership)."""
        return native().symm_view(self.base, int(offset), list(shape), dtype, self._dev)

    # -------------------------------------------------------------- errors
    def poll_error(self) -> None:
        """Raise if an earlier kernel recorded a failed wait (reads last call's copy; no sync)."""
        code = int(self._host_err[0])
        if code:
            raise RuntimeError(f"symmetric-memory collective failed on rank {self.rank}: "
                               f"{_ERR_NAMES.get(code, f'error {code}')}")
        self._host_err.copy_(self.err, non_blocking=True)

    def check(self) -> None:
        """Synchronous error check."""
        torch.cuda.synchronize(self.device)
        self._host_err.copy_(self.err)
        self.poll_error()

    # ------------------------------------------------------------- teardown
    def close(self) -> None:
        if self._closed:
            return
        C = native()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            C.symm_close(p, self._dev)
        dist.barrier(group=self.group)
        C.symm_free(self.base, self._dev)
        self._closed = True
