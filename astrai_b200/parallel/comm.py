"""Gradient exchange for data parallelism.

``GradReducer.reduce()`` averages every gradient across the data-parallel
group once per optimizer step. Backends:

* ``nccl``  - asynchronous NCCL all-reduces (AVG), one per gradient, issued
  back to back so NCCL pipelines them; the baseline path.
* ``fused`` - the framework's own all-reduce over NVLink peer memory
  (astrai_b200.parallel.symm), one kernel launch per bucket, which also
  accumulates the squared L2 norm of the reduced gradients for clipping.

Parity: replaces the bucketed DDP all-reduce of the reference
(astrai/parallel/executor.py:178-236, C4 in the collective inventory).
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn


class GradReducer:
    """Parameters flagged ``_ep_local`` (experts sharded by expert parallelism)
    are not exchanged: their gradients already sum every rank's tokens, so they
    are only scaled by 1/world (to match the mean over ranks), and their
    squared norm is summed over ranks for clipping."""

    def __init__(self, model: nn.Module, backend: str = "nccl", bucket_cap_mb: int = 256, group=None):
        self.params: List[nn.Parameter] = []
        self.ep_params: List[nn.Parameter] = []
        seen = set()
        for p in model.parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                (self.ep_params if getattr(p, "_ep_local", False) else self.params).append(p)
        self.backend = backend
        self.group = group
        self.bucket_cap = bucket_cap_mb << 20
        self._fused = None
        self.last_sumsq: Optional[torch.Tensor] = None  # set by the fused backend, consumed by clipping

    def _grads(self) -> List[torch.Tensor]:
        out = []
        for p in self.params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            out.append(p.grad)
        return out

    def _reduce_ep(self, sumsq: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        if not self.ep_params:
            return sumsq
        ws = dist.get_world_size(self.group)
        grads = []
        for p in self.ep_params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            grads.append(p.grad)
        torch._foreach_mul_(grads, 1.0 / ws)
        if sumsq is None:
            return None
        local = torch.stack([g.float().pow(2).sum() for g in grads]).sum().reshape(1)
        dist.all_reduce(local, group=self.group)
        return sumsq + local

    def reduce(self) -> Optional[torch.Tensor]:
        grads = self._grads()
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return None
        if self.backend == "fused" and grads and grads[0].is_cuda:
            if self._fused is None:
                from astrai_b200.parallel.symm import FusedAllReduce

                self._fused = FusedAllReduce(self.group)
            self.last_sumsq = self._reduce_ep(self._fused.all_reduce_mean(grads))
            return self.last_sumsq
        works = [dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.group, async_op=True)
                 if g.is_cuda else dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
                 for g in grads]
        for w in works:
            w.wait()
        if grads and not grads[0].is_cuda:  # gloo has no AVG
            ws = dist.get_world_size(self.group)
            for g in grads:
                g.div_(ws)
        self._reduce_ep(None)
        return None
