"""Expert parallelism: per-layer symmetric arenas and the dispatch layout.

Experts of a MoE layer are split over the ranks of an expert-parallel group
(``E_local = E / W`` consecutive experts per rank). Each MoE layer owns an
:class:`EPArena`: one symmetric buffer per rank (mapped into every peer)
holding the expert input block, the expert output-gradient block, the return
blocks of this rank's token slots and the epoch flags of the four exchange
phases. Token rows travel with P2P stores issued by the dispatch / return /
combine-backward kernels of ``csrc/moe.cu``; no collective library call moves
token data. The only host synchronisation per layer and step is the
all-gather of the per-expert counts (``W x E`` int32) that fixes the layout.

Layout (:class:`EPLayout`): rank r stores expert e_l's rows in
``[e_l * C_r, e_l * C_r + n_{r, e_l})`` of its input block, with the rows of
source rank q after those of ranks < q; ``C_r`` is the largest local expert
load rounded up to 128 rows, so the expert GEMMs run as batched GEMMs over
``[E_local, C_r, d]`` blocks (padding rows are zeroed in the gradient block
so they add nothing to the weight gradients).

Parity: the reference replicates every expert on every rank
(astrai/model/components/mlp.py:28-100); the layer semantics (softmax
router, top-k, renormalised weights, shared experts) are kept.
"""

from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.distributed as dist

from astrai_b200.parallel.symm import SymmetricBuffer, _align

PH_DISPATCH, PH_RETURN, PH_SCATTER_BWD, PH_RETURN_BWD = 0, 1, 2, 3


class EPGroup:
    """Process group + rank / size of expert parallelism (world 1 without distributed)."""

    def __init__(self, group=None):
        init = dist.is_available() and dist.is_initialized()
        self.group = group
        self.rank = dist.get_rank(group) if init else 0
        self.world = dist.get_world_size(group) if init else 1

    @classmethod
    def local(cls) -> "EPGroup":
        """A group of this rank alone (experts replicated, no exchange)."""
        g = cls.__new__(cls)
        g.group, g.rank, g.world = None, 0, 1
        return g

    def all_gather_counts(self, counts: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return counts.view(1, -1)
        out = torch.empty((self.world, counts.numel()), dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(out, counts.contiguous(), group=self.group)
        return out


class EPLayout:
    """Where every (source rank, expert) slot range lives; computed identically on every rank.

    Rank r's block holds its experts back to back, each padded to whole
    128-row tiles: expert e_l starts at ``starts_r[e_l]`` and has ``n_{r,e_l}``
    valid rows, the rows of source rank q after those of ranks < q. The
    grouped expert GEMMs read ``group_tile`` (the expert of each 128-row tile)
    and, for the weight gradients, ``k_start`` / ``k_count`` (padded ranges).
    """

    def __init__(self, counts_all, rank: int, e_local: int, device, row_align: int = 128):
        import numpy as np

        c = np.asarray(counts_all, dtype=np.int64)  # [W, E]
        W, E = c.shape
        self.W, self.E, self.e_local, self.rank = W, E, e_local, rank
        loads = c.sum(0).reshape(W, e_local)                       # [W, e_local] rows per expert
        padded = (loads + row_align - 1) // row_align * row_align
        starts = np.cumsum(padded, axis=1) - padded                # [W, e_local]
        self.totals = [int(x) for x in padded.sum(1)]
        before = np.cumsum(c, axis=0) - c                          # rows of earlier source ranks, per expert
        base = np.empty(E, dtype=np.int64)
        for e in range(E):
            r, el = divmod(e, e_local)
            base[e] = starts[r, el] + before[rank, e]
        self.total = self.totals[rank]
        self.n_rows_host = [int(x) for x in loads[rank]]
        tiles = np.repeat(np.arange(e_local, dtype=np.int64), padded[rank] // row_align)
        packed = np.concatenate([base, loads[rank], starts[rank], padded[rank], tiles]).astype(np.int32)
        dev = torch.tensor(packed).to(device, non_blocking=True)   # one H2D copy for every table
        self.base_row = dev[:E]
        self.n_rows = dev[E:E + e_local]
        self.starts = dev[E + e_local:E + 2 * e_local]
        self.k_count = dev[E + 2 * e_local:E + 3 * e_local]
        self.group_tile = dev[E + 3 * e_local:]
        self.max_rows = max(self.totals)


class EPArena:
    """Symmetric buffer of one MoE layer (see module docstring)."""

    def __init__(self, ep: EPGroup, d: int, tokens: int, top_k: int, n_experts: int, capacity_factor: float = 2.0,
                 device=None, wait_s: float = 20.0, min_rows: int = 0, fp8: bool = False):
        self.ep, self.d = ep, d
        self.e_local = n_experts // ep.world
        self.slots_cap = tokens * top_k
        mean = tokens * top_k * ep.world / n_experts
        c_cap = int(math.ceil(capacity_factor * mean / 128.0)) * 128 + 128
        self.rows_cap = max(self.e_local * c_cap, int(min_rows))
        W = ep.world
        o_flags = 0
        o_src = _align(4 * W * 4)
        o_xin = o_src + _align(self.rows_cap * 8)
        o_dyin = o_xin + _align(self.rows_cap * d * 2)
        o_ret = o_dyin + _align(self.rows_cap * d * 2)
        o_ret2 = o_ret + _align(self.slots_cap * d * 2)
        total = o_ret2 + _align(self.slots_cap * d * 2)
        # fp8 dispatch (opt-in): e4m3 rows and one fp32 scale per 128 columns, dequantised into xin
        self.fp8 = bool(fp8) and d % 128 == 0
        o_xin8 = o_xsc = 0
        if self.fp8:
            o_xin8 = total
            o_xsc = o_xin8 + _align(self.rows_cap * d)
            total = o_xsc + _align(self.rows_cap * (d // 128) * 4)
        self.offs = [o_flags, o_src, o_xin, o_dyin, o_ret, o_ret2, o_xin8, o_xsc]
        self.buf = SymmetricBuffer(total, ep.group, device, local_only=ep.world == 1)
        self.device = self.buf.device
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = [0, 0, 0, 0]
        self.wait_s = wait_s

    # argument prefix shared by every arena kernel binding
    def args(self):
        return (self.buf.peer_base, self.offs, self.done, self.ep.rank, self.ep.world, self.rows_cap, self.slots_cap,
                self.d, self.wait_s)

    def next_epoch(self, phase: int) -> int:
        self.epoch[phase] += 1
        return self.epoch[phase]

    def block(self, which: str, rows: int) -> torch.Tensor:
        off = self.offs[{"xin": 2, "dyin": 3, "ret": 4, "ret2": 5}[which]]
        return self.buf.local_view(off, rows * self.d * 2).view(torch.bfloat16).view(rows, self.d)

    def check(self, layout: EPLayout) -> None:
        if layout.max_rows > self.rows_cap:
            raise RuntimeError(f"expert load needs {layout.max_rows} rows per rank, the EP arena holds "
                               f"{self.rows_cap}: raise the MoE capacity factor")

    def close(self) -> None:
        self.buf.close()
