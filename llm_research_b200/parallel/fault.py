"""Host-side failure detection and fault injection.

* :class:`HeartbeatMonitor` -- every rank's background thread writes
  ``hb/<rank> = (time, epoch)`` into the process group's TCPStore every
  ``interval_s``; :meth:`live_ranks` returns the ranks whose heartbeat is
  younger than ``timeout_s``.  Nothing touches the GPU, so a stalled or dead
  rank is detected without a device fault, and the survivors can regroup at
  the next safe point (the DiLoCo outer step does).
* :class:`FaultInjector` -- test hook that makes a rank fail on the host at a
  chosen step: raise, stop heart-beating (a hang as seen from outside), or
  leave the job between steps.  It never touches the GPU.

Device-side waits of the framework's own kernels are bounded and report an
error code instead (``llm_research_b200.parallel.symm``); collectives use
short process-group timeouts.
"""

from __future__ import annotations

import os
import threading
import time
from typing import Dict, List, Optional

import torch.distributed as dist


def default_store():
    """The default process group's store (a TCPStore under torchrun / env init)."""
    from torch.distributed.distributed_c10d import _get_default_store

    return _get_default_store()


def private_store(timeout_s: float = 30.0):
    """A separate client connection to the job's TCPStore (``MASTER_ADDR``/``MASTER_PORT``).
    A store client is not safe to share between threads, so the heartbeat
    thread gets its own."""
    from datetime import timedelta

    return dist.TCPStore(os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"]),
                         is_master=False, timeout=timedelta(seconds=timeout_s), wait_for_workers=False)


class HeartbeatMonitor:
    def __init__(self, store=None, rank: Optional[int] = None, world: Optional[int] = None,
                 interval_s: float = 1.0, timeout_s: float = 10.0, prefix: str = "lrb_hb") -> None:
        self.store = store if store is not None else private_store()
        self._lock = threading.Lock()  # the beat thread and the caller share this client
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval_s = interval_s
        self.timeout_s = timeout_s
        self.prefix = prefix
        self.epoch = 0
        self._stop = threading.Event()
        self._paused = threading.Event()
        self._thread: Optional[threading.Thread] = None

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        with self._lock:
            self.store.set(self._key(self.rank), f"{time.time():.6f} {self.epoch}")

    def start(self) -> "HeartbeatMonitor":
        self.beat()

        def loop() -> None:
            while not self._stop.wait(self.interval_s):
                if not self._paused.is_set():
                    try:
                        self.beat()
                    except Exception:  # store gone: the job is ending
                        return

        self._thread = threading.Thread(target=loop, name="lrb-heartbeat", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5.0)

    def pause(self) -> None:
        """Stop beating (used by fault injection to simulate a hung rank)."""
        self._paused.set()

    def read(self) -> Dict[int, float]:
        """Last heartbeat time of every rank that ever beat."""
        out: Dict[int, float] = {}
        with self._lock:
            for r in range(self.world):
                k = self._key(r)
                try:
                    if self.store.check([k]):
                        out[r] = float(self.store.get(k).decode().split()[0])
                except Exception:
                    continue
        return out

    def live_ranks(self, now: Optional[float] = None) -> List[int]:
        now = time.time() if now is None else now
        return sorted(r for r, t in self.read().items() if now - t <= self.timeout_s)

    def wait_for_stale(self, ranks: List[int], limit_s: float) -> List[int]:
        """Block up to ``limit_s`` until each rank in ``ranks`` is either fresh or stale;
        returns the live subset at the end (used right after a peer misses a deadline)."""
        deadline = time.time() + limit_s
        while time.time() < deadline:
            hb = self.read()
            now = time.time()
            if all((r in hb) for r in ranks):
                break
            time.sleep(self.interval_s / 2)
        return [r for r in self.live_ranks() if r in ranks]


class RosterGroup:
    """Collectives over an arbitrary subset of the job's ranks, built directly on
    the job store under a caller-chosen key.  Unlike ``dist.new_group`` it needs
    no call from ranks outside the subset and no agreement on how many groups
    each rank created before, so survivors of a failure (and a rank that
    rejoins) can form it at a safe point.  Gloo for CPU tensors, NCCL for CUDA."""

    def __init__(self, ranks: List[int], key: str, device) -> None:
        import torch

        self.ranks = list(ranks)
        self.index = self.ranks.index(dist.get_rank())
        self.size = len(self.ranks)
        store = dist.PrefixStore(f"lrb_roster/{key}", default_store())
        if torch.device(device).type == "cuda":
            self.pg = dist.ProcessGroupNCCL(store, self.index, self.size)
        else:
            self.pg = dist.ProcessGroupGloo(store, self.index, self.size)

    def all_reduce(self, t) -> None:
        self.pg.allreduce([t]).wait()

    def broadcast(self, t, src: int) -> None:
        self.pg.broadcast(t, self.ranks.index(src)).wait()

    def all_gather(self, outs, t) -> None:
        self.pg.allgather([outs], [t]).wait()


class FaultInjector:
    """``LRB_FAULT="<rank>:<step>:<mode>"`` with mode ``raise`` | ``hang`` | ``leave``."""

    def __init__(self, spec: Optional[str] = None, rank: Optional[int] = None) -> None:
        spec = spec if spec is not None else os.environ.get("LRB_FAULT", "")
        self.rank = dist.get_rank() if rank is None else rank
        self.plan: Dict[int, str] = {}
        for item in filter(None, (s.strip() for s in spec.split(","))):
            r, step, mode = item.split(":")
            if int(r) == self.rank:
                self.plan[int(step)] = mode

    def check(self, step: int, monitor: Optional[HeartbeatMonitor] = None) -> Optional[str]:
        """Call between steps.  Returns ``"leave"`` when this rank should exit the
        training loop now; raises for ``raise``; stops heart-beating for ``hang``."""
        mode = self.plan.get(step)
        if mode is None:
            return None
        if mode == "raise":
            raise RuntimeError(f"injected fault on rank {self.rank} at step {step}")
        if mode == "hang":
            if monitor is not None:
                monitor.pause()
            return "leave"
        return "leave"
