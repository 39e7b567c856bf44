"""Expert parallelism: per-layer symmetric arenas and the device-side dispatch layout.

Experts of a MoE layer are split over the ranks of an expert-parallel group
(``E_local = E / W`` consecutive experts per rank). Each MoE layer owns an
:class:`EPArena`: one symmetric buffer per rank (mapped into every peer)
holding the arrival counters of the five exchange phases, the routed-slot
counts of every rank, the expert input block, the expert output-gradient
block, the return blocks of this rank's token slots. Token rows travel with
P2P stores issued by the dispatch / return / combine-backward kernels of
``csrc/moe.cu``; no collective library call moves token data, and nothing is
read back to the host: the counts exchange and the layout run in one kernel
(``ep_layout``), the grouped GEMMs skip the unused tiles of the
capacity-sized blocks, and phase completion is counted on the device. A MoE
layer's forward and backward can therefore be captured in a CUDA graph.

Layout (:class:`EPLayout`, device tables written by ``ep_layout``): rank r
stores expert e_l's rows in ``[start_{r,e_l}, start_{r,e_l} + n_{r,e_l})`` of
its input block, with the rows of source rank q after those of ranks < q;
each expert's range is padded to whole 128-row tiles and the experts of a rank
follow each other from row 0, so the expert GEMMs run as grouped GEMMs over
the rank's block (``group_tile[t]`` = expert of tile t, -1 for tiles past the
block's live rows). Padding rows are zeroed in the gradient block so they add
nothing to the weight gradients. The block is sized for ``capacity_factor``
times the mean expert load; a load beyond it is reported through the device
error word (kErrBadArg) and its rows are dropped rather than written out of
bounds.

Parity: the reference replicates every expert on every rank
(astrai/model/components/mlp.py:28-100); the layer semantics (softmax
router, top-k, renormalised weights, shared experts) are kept.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from astrai_b200.parallel.symm import SymmetricBuffer, _align

PH_DISPATCH, PH_RETURN, PH_SCATTER_BWD, PH_RETURN_BWD, PH_COUNTS = 0, 1, 2, 3, 4
N_PHASES = 5


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


class EPLayout:
    """Device tables of one dispatch layout, rewritten by every :meth:`EPArena.compute_layout`.

    ``base_row [E]``: first row of this rank's slots in expert e's block on its owner;
    ``n_rows / starts / k_count [E_local]``: live rows, first row and padded rows of this rank's
    experts; ``group_tile [rows_cap / 128]``; ``total [1]``: live (padded) rows of this rank's block.
    ``rows`` is the static block size the buffers and GEMMs are shaped for."""

    def __init__(self, n_experts: int, e_local: int, rows_cap: int, device):
        i32 = dict(device=device, dtype=torch.int32)
        self.E, self.e_local, self.rows = n_experts, e_local, rows_cap
        self.base_row = torch.zeros(n_experts, **i32)
        self.n_rows = torch.zeros(e_local, **i32)
        self.starts = torch.zeros(e_local, **i32)
        self.k_count = torch.zeros(e_local, **i32)
        self.group_tile = torch.full((rows_cap // 128,), -1, **i32)
        self.total = torch.zeros(1, **i32)


class EPArena:
    """Symmetric buffer of one MoE layer (see module docstring)."""

    def __init__(self, ep: EPGroup, d: int, tokens: int, top_k: int, n_experts: int, capacity_factor: float = 2.0,
                 device=None, wait_s: float = 20.0, min_rows: int = 0, fp8: bool = False):
        self.ep, self.d = ep, d
        self.n_experts = n_experts
        self.e_local = n_experts // ep.world
        self.slots_cap = tokens * top_k
        mean = tokens * top_k * ep.world / n_experts
        c_cap = int(math.ceil(capacity_factor * mean / 128.0)) * 128 + 128
        self.rows_cap = max(self.e_local * c_cap, (int(min_rows) + 127) // 128 * 128)
        W = ep.world
        o_flags = 0
        o_counts = _align(N_PHASES * W * 4)
        o_src = o_counts + _align(W * n_experts * 4)
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
        self.offs = [o_flags, o_src, o_xin, o_dyin, o_ret, o_ret2, o_xin8, o_xsc, o_counts]
        # zeroed: arrival counters start at 0, and padding rows of the blocks hold finite values
        self.buf = SymmetricBuffer(total, ep.group, device, local_only=ep.world == 1, zero=True)
        self.device = self.buf.device
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.expect = torch.zeros(N_PHASES, dtype=torch.int32, device=self.device)  # rounds waited per phase
        self.wait_s = wait_s
        self.layout = EPLayout(n_experts, self.e_local, self.rows_cap, self.device)

    # argument prefix shared by every arena kernel binding
    def args(self):
        return (self.buf.peer_base, self.offs, self.done, self.expect, self.ep.rank, self.ep.world, self.rows_cap,
                self.slots_cap, self.d, self.wait_s)

    def compute_layout(self, counts: torch.Tensor) -> EPLayout:
        """Exchange this rank's per-expert slot counts and rebuild :attr:`layout` (device only)."""
        from astrai_b200.ops._ext import native

        L = self.layout
        native().ep_layout(*self.args(), counts, self.e_local, L.base_row, L.n_rows, L.starts, L.k_count,
                           L.group_tile, L.total)
        return L

    def block(self, which: str, rows: int) -> torch.Tensor:
        off = self.offs[{"xin": 2, "dyin": 3, "ret": 4, "ret2": 5}[which]]
        return self.buf.local_view(off, rows * self.d * 2).view(torch.bfloat16).view(rows, self.d)

    def close(self) -> None:
        self.buf.close()
