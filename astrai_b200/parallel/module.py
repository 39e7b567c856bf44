"""Tensor-parallel linear layers.

API parity with astrai/parallel/module.py:10-115: ``RowParallelLinear``
(input features sharded, partial products summed over the group) and
``ColumnParallelLinear`` (output features sharded, optional all-gather of
the shards), constructed with ``(process_group, in_features, out_features,
bias, reduce_results / gather_results)``; ``load_state_dict`` takes the FULL
weight / bias and keeps this rank's slice.

Differences: the local products run on the framework's GEMM (CUDA bf16) or
``F.linear``, and the collectives are autograd functions, so the layers train
correctly (the backward of the sum is the identity on every rank, the
backward of the gather is the rank's slice of the output gradient); the
reference calls ``dist.all_reduce`` / ``dist.all_gather`` outside autograd.
"""

from __future__ import annotations

from typing import Dict

import torch
import torch.distributed as dist
import torch.nn as nn
from torch import Tensor

from astrai_b200.ops.gemm import linear


class _AllReduceSum(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        y = x.contiguous().clone()
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


class _AllGatherLast(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, rank, world):
        x = x.contiguous()
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x, group=group)
        ctx.rank, ctx.width = rank, x.shape[-1]
        return torch.cat(parts, dim=-1)

    @staticmethod
    def backward(ctx, g):
        s = ctx.rank * ctx.width
        return g[..., s:s + ctx.width].contiguous(), None, None, None


class ParallelModel(nn.Module):
    def __init__(self, process_group=None):
        super().__init__()
        self.process_group = process_group
        self.rank = dist.get_rank(process_group)
        self.world_size = dist.get_world_size(process_group)


def _matmul(x: Tensor, w: Tensor) -> Tensor:
    return linear(x, w) if x.is_cuda and x.dtype == torch.bfloat16 else torch.nn.functional.linear(x, w)


class RowParallelLinear(ParallelModel):
    def __init__(self, process_group, in_features: int, out_features: int, bias: bool = True,
                 reduce_results: bool = True):
        super().__init__(process_group)
        if in_features % self.world_size:
            raise ValueError(f"in_features must be divisible by world_size. Got {in_features} and {self.world_size}")
        self.in_features, self.out_features = in_features, out_features
        self.in_features_per_rank = in_features // self.world_size
        self.reduce_results = reduce_results
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_rank))
        nn.init.normal_(self.weight, std=0.02)
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

    def forward(self, input: Tensor) -> Tensor:
        """``input`` holds this rank's slice of the input features."""
        out = _matmul(input, self.weight)
        if self.reduce_results and self.world_size > 1:
            out = _AllReduceSum.apply(out, self.process_group)
        return out + self.bias if self.bias is not None else out

    def load_state_dict(self, state_dict: Dict[str, Tensor], strict: bool = True, assign: bool = False):
        s = self.rank * self.in_features_per_rank
        with torch.no_grad():
            self.weight.copy_(state_dict["weight"][:, s:s + self.in_features_per_rank])
            if self.bias is not None:
                self.bias.copy_(state_dict["bias"])


class ColumnParallelLinear(ParallelModel):
    def __init__(self, process_group, in_features: int, out_features: int, bias: bool = True,
                 gather_results: bool = True):
        super().__init__(process_group)
        if out_features % self.world_size:
            raise ValueError(f"out_features must be divisible by world_size. Got {out_features} and {self.world_size}")
        self.in_features, self.out_features = in_features, out_features
        self.out_features_per_rank = out_features // self.world_size
        self.gather_results = gather_results
        self.weight = nn.Parameter(torch.empty(self.out_features_per_rank, in_features))
        nn.init.normal_(self.weight, std=0.02)
        self.bias = nn.Parameter(torch.zeros(self.out_features_per_rank)) if bias else None

    def forward(self, input: Tensor) -> Tensor:
        out = _matmul(input, self.weight)
        if self.bias is not None:
            out = out + self.bias
        if self.gather_results and self.world_size > 1:
            out = _AllGatherLast.apply(out, self.process_group, self.rank, self.world_size)
        return out

    def load_state_dict(self, state_dict: Dict[str, Tensor], strict: bool = True, assign: bool = False):
        s = self.rank * self.out_features_per_rank
        with torch.no_grad():
            self.weight.copy_(state_dict["weight"][s:s + self.out_features_per_rank])
            if self.bias is not None:
                self.bias.copy_(state_dict["bias"][s:s + self.out_features_per_rank])
