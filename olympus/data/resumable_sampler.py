"""A distributed sampler whose position inside an epoch can be saved and restored
(an extension: the reference's checkpoints keep the epoch only, so a resumed
run starts that epoch over and sees some samples twice).

Every epoch draws one permutation of the dataset from ``seed + epoch`` (the
same on every rank), drops the tail that does not divide by the number of
replicas, and gives rank ``r`` the entries ``r, r + R, r + 2R, ...``.  The
trainer reports the samples it has consumed with :meth:`advance`;
:meth:`state_dict` / :meth:`load_state_dict` carry ``(epoch, consumed)``, and
the first epoch iterated after a restore skips the consumed samples, so the
resumed run sees exactly the samples an uninterrupted one would.
"""

from __future__ import annotations

from typing import Any, Dict, Iterator

import torch
from torch.utils.data import Sampler


class ResumableDistributedSampler(Sampler):
    def __init__(self, dataset_len: int, num_replicas: int = 1, rank: int = 0, shuffle: bool = True,
                 seed: int = 0) -> None:
        if not 0 <= rank < num_replicas:
            raise ValueError(f"rank {rank} outside [0, {num_replicas})")
        self.n = int(dataset_len)
        self.num_replicas = num_replicas
        self.rank = rank
        self.shuffle = shuffle
        self.seed = seed
        self.epoch = 0
        self.consumed = 0  # samples of this rank consumed in ``epoch``
        self.num_samples = self.n // num_replicas

    def set_epoch(self, epoch: int) -> None:
        if epoch != self.epoch:
            self.epoch = epoch
            self.consumed = 0

    def advance(self, samples: int) -> None:
        """Record ``samples`` more samples of this rank as consumed (one optimizer micro-step)."""
        self.consumed = min(self.consumed + int(samples), self.num_samples)

    def _indices(self) -> torch.Tensor:
        if self.shuffle:
            g = torch.Generator().manual_seed(self.seed + self.epoch)
            order = torch.randperm(self.n, generator=g)
        else:
            order = torch.arange(self.n)
        order = order[: self.num_samples * self.num_replicas]
        return order[self.rank::self.num_replicas]

    def __iter__(self) -> Iterator[int]:
        return iter(self._indices()[self.consumed:].tolist())

    def __len__(self) -> int:
        return self.num_samples - self.consumed

    def state_dict(self) -> Dict[str, Any]:
        return {"epoch": self.epoch, "consumed": self.consumed, "seed": self.seed,
                "num_replicas": self.num_replicas}

    def load_state_dict(self, state: Dict[str, Any]) -> None:
        self.epoch = int(state["epoch"])
        self.seed = int(state.get("seed", self.seed))
        # a different world size splits the permutation differently: restart the epoch
        same_split = int(state.get("num_replicas", self.num_replicas)) == self.num_replicas
        self.consumed = int(state["consumed"]) if same_split else 0
