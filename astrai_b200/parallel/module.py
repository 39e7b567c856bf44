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

``ColumnParallelLinear(..., fused=True)`` (CUDA, bf16, no bias, ranks on one NVLink
domain) replaces "GEMM, then all-gather" by :class:`GatherGemm`: ONE GEMM kernel per rank
whose epilogue stores every output tile into every rank's copy of the gathered output
over NVLink peer memory, so the transfer overlaps the remaining tiles' math.
``RowParallelLinear(..., fused=True)`` replaces "GEMM, then all-reduce" by
:class:`ReduceGemm`: the GEMM's epilogue pushes the rows other ranks own into their receive
slots as tiles finish (a reduce-scatter overlapped with the GEMM), then one kernel per rank
sums its rows and writes them into every rank's output (the all-gather half).
"""

from __future__ import annotations

from typing import Dict

import torch
import torch.distributed as dist
import torch.nn as nn
from torch import Tensor

from astrai_b200.ops.gemm import linear
from astrai_b200.parallel.symm import SymmetricBuffer, _align


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


class GatherGemm:
    """``y[M, world*n] = all_gather_columns(x[M, K] @ w[n, K]^T)`` as one fused kernel per rank.

    The gathered output lives in a symmetric buffer (same offset on every rank, each rank's copy
    mapped into every rank). Call ``e`` on every rank:

    1. wait (bounded) until every peer has copied call ``e-1``'s result out of its buffer
       (flag row 1), so no peer's stores of call ``e`` can overwrite data still being read;
    2. ``gemm_gather``: the GEMM writes its column block into every rank's copy; its last CTA
       raises this rank's flag in row 0 of every peer;
    3. wait (bounded) for row 0 of every peer, copy the gathered result out, raise row 1.

    Every rank must make the same calls with the same shapes (as with any collective).
    """

    def __init__(self, group=None, wait_s: float = 20.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.wait_s = wait_s
        self.buf: SymmetricBuffer = None
        self.cap = 0
        self.epoch = 0

    def _ensure(self, nbytes: int, dev: torch.device) -> None:
        if self.buf is not None and self.cap >= nbytes:
            return
        if self.buf is not None:
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.group)
            self.buf.close()
        self.flag_off = _align(nbytes)
        self.done_off = self.flag_off + _align(4 * 2 * self.world)
        self.buf = SymmetricBuffer(self.done_off + 256, self.group, dev)
        self.buf.local_view(self.flag_off, self.done_off + 256 - self.flag_off).zero_()
        self.deltas = [self.buf.ptrs[q] - self.buf.ptrs[self.rank] for q in range(self.world) if q != self.rank]
        self.raise_done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.cap, self.epoch = nbytes, 0
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def __call__(self, x: Tensor, w: Tensor) -> Tensor:
        from astrai_b200.ops._ext import native

        C = native()
        M, n = x.shape[0], w.shape[0]
        Nt = n * self.world
        dev = x.device
        self._ensure(M * Nt * 2, dev)
        full = self.buf.local_view(0, M * Nt * 2).view(torch.bfloat16).view(M, Nt)
        flags = self.buf.local_ptr + self.flag_off
        if self.epoch > 0:
            C.peer_flags_wait(flags + 4 * self.world, dev.index, self.rank, self.world, 1, self.epoch, self.wait_s)
        self.epoch += 1
        C.gemm_gather(x, w, full[:, self.rank * n:(self.rank + 1) * n], self.deltas, flags + 4 * self.rank,
                      self.buf.local_ptr + self.done_off, self.epoch)
        C.peer_flags_wait(flags, dev.index, self.rank, self.world, 1, self.epoch, self.wait_s)
        y = full.clone()
        # this rank is done reading call `epoch`: raise its flag in row 1 on every peer
        C.muon_apply_peers(None, None, self.buf.peer_base, None, 0, 1, 1, False, 1.0, 0.0, self.rank, self.world,
                           self.flag_off, 1, self.epoch, self.raise_done)
        return y

    def close(self) -> None:
        if self.buf is not None:
            self.buf.close()
            self.buf = None


class ReduceGemm:
    """``y[M, N] = sum over ranks of x_r[M, K_r] @ w_r[N, K_r]^T`` (the row-parallel linear's
    all-reduce), fused with the GEMM.

    Rows are owned in blocks of ``rpo = ceil(M / world)``. Call ``e`` on every rank:

    1. wait until every peer consumed call ``e-1`` (flag row 2): its receive slots and output
       are free again;
    2. the GEMM computes the partial product into ``part``; as each tile finishes, its rows owned
       by other ranks are pushed into their receive slots over NVLink; the last CTA raises this
       rank's flag in row 0 of every peer;
    3. wait for row 0 of every peer (all partials of this rank's rows are here), then
       ``row_reduce_bcast`` sums this rank's rows in fp32 and writes them into every rank's
       output; its last CTA raises row 1 on every peer;
    4. wait for row 1 of every peer, copy the output out, raise row 2.
    """

    def __init__(self, group=None, wait_s: float = 20.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.wait_s = wait_s
        self.buf: SymmetricBuffer = None
        self.key = None
        self.epoch = 0

    def _ensure(self, M: int, N: int, dev: torch.device) -> None:
        if self.key == (M, N):
            return
        if self.buf is not None:
            torch.cuda.synchronize(dev)
            dist.barrier(group=self.group)
            self.buf.close()
        W = self.world
        self.rpo = -(-M // W)
        part = _align(M * N * 2)
        recv = _align(W * self.rpo * N * 2)
        out = _align(M * N * 2)
        self.off_part, self.off_recv, self.off_out = 0, part, part + recv
        self.off_flag = part + recv + out
        self.off_done = self.off_flag + _align(4 * 3 * W)
        self.buf = SymmetricBuffer(self.off_done + 256, self.group, dev)
        self.buf.local_view(self.off_flag, self.off_done + 256 - self.off_flag).zero_()
        self.rank_deltas = [self.buf.ptrs[q] - self.buf.ptrs[self.rank] for q in range(W)]
        self.peer_deltas = [d for q, d in enumerate(self.rank_deltas) if q != self.rank]
        self.raise_done = torch.zeros(1, dtype=torch.int32, device=dev)
        self.key, self.epoch = (M, N), 0
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def __call__(self, x: Tensor, w: Tensor) -> Tensor:
        from astrai_b200.ops._ext import native

        C = native()
        M, N = x.shape[0], w.shape[0]
        dev = x.device
        self._ensure(M, N, dev)
        W, r, base = self.world, self.rank, self.buf.local_ptr
        part = self.buf.local_view(self.off_part, M * N * 2).view(torch.bfloat16).view(M, N)
        out = self.buf.local_view(self.off_out, M * N * 2).view(torch.bfloat16).view(M, N)
        flags = base + self.off_flag
        if self.epoch > 0:
            C.peer_flags_wait(flags + 8 * W, dev.index, r, W, 1, self.epoch, self.wait_s)
        self.epoch += 1
        C.gemm_gather(x, w, part, self.peer_deltas, flags + 4 * r, base + self.off_done, self.epoch,
                      scatter_rpo=self.rpo, scatter_rank=r, scatter_recv_off=self.off_recv - self.off_part,
                      rank_deltas=self.rank_deltas)
        C.peer_flags_wait(flags, dev.index, r, W, 1, self.epoch, self.wait_s)
        C.row_reduce_bcast(base + self.off_part, base + self.off_recv, base + self.off_out, N, M, N, r, W, self.rpo,
                           self.rank_deltas, flags + 4 * W + 4 * r, self.epoch, base + self.off_done + 64, dev.index)
        C.peer_flags_wait(flags + 4 * W, dev.index, r, W, 1, self.epoch, self.wait_s)
        y = out.clone()
        C.muon_apply_peers(None, None, self.buf.peer_base, None, 0, 1, 1, False, 1.0, 0.0, r, W, self.off_flag, 2,
                           self.epoch, self.raise_done)
        return y

    def close(self) -> None:
        if self.buf is not None:
            self.buf.close()
            self.buf = None
            self.key = None


class _ReduceLinearFn(torch.autograd.Function):
    """Forward through :class:`ReduceGemm`; the backward of the sum is the identity on every rank."""

    @staticmethod
    def forward(ctx, x2, w, rg):
        ctx.save_for_backward(x2, w)
        return rg(x2, w)

    @staticmethod
    def backward(ctx, g):
        from astrai_b200.ops._ext import native

        x2, w = ctx.saved_tensors
        g = g.contiguous()
        C = native()
        dx = torch.empty_like(x2)
        C.gemm(g, w, dx, None, 0, 1)   # [M, N] @ [N, K_r]
        dw = torch.empty_like(w)
        C.gemm(g, x2, dw, None, 1, 1)  # [M, N]^T @ [M, K_r]
        return dx, dw, None


class _GatherLinearFn(torch.autograd.Function):
    """Forward through :class:`GatherGemm`; backward on this rank's column slice of the gradient."""

    @staticmethod
    def forward(ctx, x2, w, gg, rank):
        ctx.save_for_backward(x2, w)
        ctx.rank = rank
        return gg(x2, w)

    @staticmethod
    def backward(ctx, g):
        from astrai_b200.ops._ext import native

        x2, w = ctx.saved_tensors
        n = w.shape[0]
        gl = g[:, ctx.rank * n:(ctx.rank + 1) * n].contiguous()
        C = native()
        dx = torch.empty_like(x2)
        C.gemm(gl, w, dx, None, 0, 1)   # [M, n] @ [n, K]
        dw = torch.empty_like(w)
        C.gemm(gl, x2, dw, None, 1, 1)  # [M, n]^T @ [M, K]
        return dx, dw, None, None


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
                 reduce_results: bool = True, fused: bool = False):
        super().__init__(process_group)
        self.fused = fused
        self._rg = None
        if in_features % self.world_size:
            raise ValueError(f"in_features must be divisible by world_size. Got {in_features} and {self.world_size}")
        self.in_features, self.out_features = in_features, out_features
        self.in_features_per_rank = in_features // self.world_size
        self.reduce_results = reduce_results
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_rank))
        nn.init.normal_(self.weight, std=0.02)
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None

    def _fused_ok(self, x: Tensor) -> bool:
        return (self.fused and self.reduce_results and self.world_size > 1 and x.is_cuda
                and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16
                and self.in_features_per_rank % 8 == 0 and self.out_features % 8 == 0)

    def forward(self, input: Tensor) -> Tensor:
        """``input`` holds this rank's slice of the input features."""
        if self._fused_ok(input):
            if self._rg is None:
                self._rg = ReduceGemm(self.process_group)
            x2 = input.reshape(-1, self.in_features_per_rank).contiguous()
            out = _ReduceLinearFn.apply(x2, self.weight, self._rg).view(*input.shape[:-1], self.out_features)
            return out + self.bias if self.bias is not None else out
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
                 gather_results: bool = True, fused: bool = False):
        super().__init__(process_group)
        self.fused = fused
        self._gg = None
        if out_features % self.world_size:
            raise ValueError(f"out_features must be divisible by world_size. Got {out_features} and {self.world_size}")
        self.in_features, self.out_features = in_features, out_features
        self.out_features_per_rank = out_features // self.world_size
        self.gather_results = gather_results
        self.weight = nn.Parameter(torch.empty(self.out_features_per_rank, in_features))
        nn.init.normal_(self.weight, std=0.02)
        self.bias = nn.Parameter(torch.zeros(self.out_features_per_rank)) if bias else None

    def _fused_ok(self, x: Tensor) -> bool:
        return (self.fused and self.gather_results and self.world_size > 1 and self.bias is None and x.is_cuda
                and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16 and self.in_features % 8 == 0
                and self.out_features_per_rank % 8 == 0)

    def forward(self, input: Tensor) -> Tensor:
        if self._fused_ok(input):
            if self._gg is None:
                self._gg = GatherGemm(self.process_group)
            x2 = input.reshape(-1, self.in_features).contiguous()
            out = _GatherLinearFn.apply(x2, self.weight, self._gg, self.rank)
            return out.view(*input.shape[:-1], self.out_features)
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
