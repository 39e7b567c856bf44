"""Resumable distributed sampler.

The sample order is part of the checkpoint contract (a resumed run must see
exactly the samples the original run had not consumed), so the ordering
rules are those of the reference (astrai/dataset/sampler.py:58-73): a
permutation drawn with seed ``seed + epoch``, padded by repeating its head up
to a multiple of the world size (unless ``drop_last``), rank ``r`` taking
every ``world``-th index starting at ``r``, and iteration resuming at
``start_iter`` within the rank's share.
"""

from __future__ import annotations

from typing import Iterator, List, Optional

import torch
import torch.distributed as dist
from torch.utils.data import Dataset, Sampler


class RDSampler(Sampler[int]):
    def __init__(self, data_source: Dataset, start_epoch: int = 0, start_iter: int = 0, seed: int = 42,
                 drop_last: bool = False, shuffle: bool = True, process_group: Optional[dist.ProcessGroup] = None):
        self.epoch = start_epoch
        self.seed = seed
        self.num_samples = len(data_source)
        if process_group is not None:
            self.rank, self.num_replicas = dist.get_rank(process_group), dist.get_world_size(process_group)
        elif dist.is_available() and dist.is_initialized():
            self.rank, self.num_replicas = dist.get_rank(), dist.get_world_size()
        else:
            self.rank, self.num_replicas = 0, 1
        self.drop_last = drop_last
        self.shuffle = shuffle
        pad = 0 if drop_last else self.num_replicas - 1
        self.num_samples_per_replica = max(1, (self.num_samples + pad) // self.num_replicas)
        self.total_size = self.num_samples_per_replica * self.num_replicas
        self.iter = start_iter % self.num_samples_per_replica
        self._indices: Optional[List[int]] = None

    def _order(self) -> List[int]:
        if self.shuffle:
            g = torch.Generator()
            g.manual_seed(self.seed + self.epoch)
            idx = torch.randperm(self.num_samples, generator=g).tolist()
        else:
            idx = list(range(self.num_samples))
        if not self.drop_last and len(idx) < self.total_size:
            idx = idx + idx[: self.total_size - len(idx)]
        return idx[self.rank: self.total_size: self.num_replicas]

    def __iter__(self) -> Iterator[int]:
        if self._indices is None:
            self.iter %= self.num_samples_per_replica
            self._indices = self._order()[self.iter:]
        for i in self._indices:
            self.iter += 1
            yield i
        self.epoch += 1
        self._indices = None
        self.iter %= self.num_samples_per_replica

    def __len__(self) -> int:
        return max(self.num_samples_per_replica - self.iter, 0)
