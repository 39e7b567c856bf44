"""Fully sharded data parallelism over NVLink peer memory (``fsdp2`` with ``comm_backend="fused"``).

The reference shards with torch ``fully_shard`` on every child module
(astrai/parallel/executor.py:316-407): every parameter is split evenly over the
ranks as a DTensor, each wrapped module all-gathers its parameters before its
forward and backward, and reduce-scatters its gradients after the backward, all
through NCCL. Two consequences on this hardware: ``torch.optim.Muon`` then runs
Newton-Schulz on row shards instead of whole matrices (a different update), and
every micro-batch repeats the all-gathers.

Here the unit of sharding is the whole tensor:

* :class:`ShardPlan` gives every parameter ONE owner rank (largest first, to the
  least-loaded rank; identical on every rank). The owner keeps the parameter in
  a symmetric (CUDA IPC) pool that peers read over NVLink, and only the owner
  holds its optimizer state and steps it. Newton-Schulz therefore sees whole
  matrices, and AdamW, being elementwise, does not care.
* Gradients accumulate into full-size bf16 buffers that also live in a
  symmetric pool, at the same offset on every rank. After the last micro-batch
  every rank announces its gradients (a release flag on every peer); each owner
  then pulls its parameters' gradients from all ranks and reduces them in one
  kernel (``fsdp_reduce``: fp32 sum, 1/world scale, bf16 mean written in place,
  squared norm for clipping). The reduce-scatter of the reference becomes a
  reduce-to-owner fused with the cast, scale and norm, once per optimizer step.
* After the owners' optimizer step every rank raises a publish flag; each rank
  then copies the parameters it does not own from their owners with the copy
  engines (``cudaMemcpyAsync`` from the peer mapping on a side stream; no SM
  time), unit by unit, and the next forward waits on each unit's copy only
  when it reaches that unit. One gather per optimizer step, not one per
  micro-batch, overlapped with the forward of the units before it.

Non-owned parameters keep a local, replicated copy between the gathers (the
``reshard_after_forward=False`` memory point of FSDP2: parameters whole,
gradients whole, optimizer state and the update sharded). Every wait is bounded
on the device (``peer_flags_wait``) and raises the extension's error word.
"""

from __future__ import annotations

import logging
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

logger = logging.getLogger(__name__)

_ALIGN = 256


def _align(x: int) -> int:
    return (x + _ALIGN - 1) // _ALIGN * _ALIGN


class ShardPlan:
    """Owner of every parameter and the byte layouts of the parameter and gradient pools.

    ``params``: ``(name, nbytes)`` in model order, the same on every rank. Owners are assigned
    largest tensor first, each to the rank with the fewest bytes so far (lowest rank on ties),
    so the plan is a pure function of the sizes and the world size.
    """

    def __init__(self, params: Sequence[Tuple[str, int]], world: int):
        if world < 1:
            raise ValueError("world must be >= 1")
        self.world = world
        self.names = [n for n, _ in params]
        self.nbytes = [int(b) for _, b in params]
        n = len(params)
        order = sorted(range(n), key=lambda i: (-self.nbytes[i], i))
        self.load = [0] * world
        self.owner = [0] * n
        for i in order:
            r = min(range(world), key=lambda q: (self.load[q], q))
            self.owner[i] = r
            self.load[r] += self.nbytes[i]
        # gradient pool: every parameter in model order (same offsets on every rank)
        self.grad_off: List[int] = []
        off = 0
        for b in self.nbytes:
            self.grad_off.append(off)
            off = _align(off + b)
        self.grad_bytes = off
        # parameter pool: each rank's owned parameters in model order
        self.param_off = [0] * n
        used = [0] * world
        for i, b in enumerate(self.nbytes):
            r = self.owner[i]
            self.param_off[i] = used[r]
            used[r] = _align(used[r] + b)
        self.pool_used = used
        self.param_bytes = max(used) if used else 0

    def owned(self, rank: int) -> List[int]:
        return [i for i in range(len(self.names)) if self.owner[i] == rank]

    def imbalance(self) -> float:
        """max over ranks of owned bytes / mean owned bytes (1.0 = perfect)."""
        total = sum(self.load)
        return max(self.load) * self.world / total if total else 1.0


def model_units(model: nn.Module) -> List[nn.Module]:
    """The wrapping units of the reference's FSDP2 executor: every direct child of the model, and
    every element of a direct ``nn.ModuleList`` child."""
    units: List[nn.Module] = []
    for child in model.children():
        if isinstance(child, nn.ModuleList):
            units.extend(child)
        elif any(True for _ in child.parameters()):
            units.append(child)
    return units


class FusedFSDP:
    """Runtime of the fused FSDP for one model (CUDA, bf16 parameters, world > 1)."""

    READY, REDUCED, PUBLISHED = 0, 1, 2
    ROWS = 3

    def __init__(self, model: nn.Module, group=None, wait_s: float = 60.0, broadcast: bool = True):
        from astrai_b200.ops._ext import native
        from astrai_b200.parallel.symm import SymmetricBuffer

        self.C = native()
        self.model = model
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.wait_s = float(wait_s)
        seen, named = set(), []
        for name, p in model.named_parameters():
            if p.requires_grad and id(p) not in seen:
                seen.add(id(p))
                named.append((name, p))
        bad = [n for n, p in named if not (p.is_cuda and p.dtype == torch.bfloat16 and p.is_contiguous()
                                          and p.numel() % 8 == 0)]
        if bad:
            raise ValueError(f"fused FSDP needs contiguous bf16 CUDA parameters with numel % 8 == 0: {bad[:3]}")
        self.names = [n for n, _ in named]
        self.params = [p for _, p in named]
        self.device = self.params[0].device
        if broadcast:
            with torch.no_grad():
                for t in list(model.parameters()) + list(model.buffers()):
                    dist.broadcast(t.data, src=0, group=group)
        # parameters the kernels pack into one buffer (q|k|v, up|gate, stacked experts) stay together:
        # pack them now, then shard by storage region (one owner and one contiguous pool range each)
        from astrai_b200.ops.gemm import pack_params

        for m in model.modules():
            groups = m.packed_groups() if hasattr(m, "packed_groups") else []
            for grp in groups:
                if len(grp) > 1 and all(p.requires_grad for p in grp):
                    pack_params(grp)
        regions: Dict[int, List[int]] = {}
        for i, p in enumerate(self.params):
            regions.setdefault(p.untyped_storage().data_ptr(), []).append(i)
        self.regions: List[List[int]] = []
        for members in regions.values():
            members.sort(key=lambda i: self.params[i].data_ptr())
            lo = self.params[members[0]].data_ptr()
            hi = max(self.params[i].data_ptr() + self.params[i].numel() * 2 for i in members)
            if hi - lo != sum(self.params[i].numel() * 2 for i in members):
                raise ValueError("fused FSDP: parameters sharing a storage must tile it contiguously")
            self.regions.append(members)
        self.regions.sort(key=lambda mem: mem[0])  # model order
        rbytes = [sum(self.params[i].numel() * 2 for i in mem) for mem in self.regions]
        self.plan = ShardPlan([(self.names[mem[0]], b) for mem, b in zip(self.regions, rbytes)], self.world)
        self.flag_off = _align(self.plan.param_bytes)
        self.pbuf = SymmetricBuffer(self.flag_off + _align(4 * self.ROWS * self.world), group, self.device, zero=True)
        self.gbuf = SymmetricBuffer(max(self.plan.grad_bytes, _ALIGN), group, self.device, zero=True)
        own = set(self.plan.owned(self.rank))
        self.owned = [self.params[i] for r in sorted(own) for i in self.regions[r]]
        self._own_ids = {id(p) for p in self.owned}
        self._grad_views: List[Optional[torch.Tensor]] = [None] * len(self.params)
        with torch.no_grad():
            for r, mem in enumerate(self.regions):
                pool = self.pbuf.local_view(self.plan.param_off[r], rbytes[r]) if r in own else None
                gview = self.gbuf.local_view(self.plan.grad_off[r], rbytes[r])
                off = 0
                for i in mem:
                    p = self.params[i]
                    nb = p.numel() * 2
                    if pool is not None:  # the owner keeps the region in the symmetric pool (peers read it)
                        view = pool[off:off + nb].view(p.dtype).view(p.shape)
                        view.copy_(p.data)
                        p.data = view
                    self._grad_views[i] = gview[off:off + nb].view(p.dtype).view(p.shape)
                    off += nb
        self._attach_grads()
        vecs = [0]
        for r in sorted(own):
            vecs.append(vecs[-1] + rbytes[r] // 16)
        self.total_vec = vecs[-1]
        self.seg_off = torch.tensor([self.plan.grad_off[r] for r in sorted(own)], dtype=torch.int64,
                                    device=self.device)
        self.seg_vec = torch.tensor(vecs, dtype=torch.int64, device=self.device)
        self.sumsq = torch.zeros(1, dtype=torch.float32, device=self.device)
        # gathers: the regions this rank does not own, grouped by wrapping unit in forward order
        unit_of: Dict[int, int] = {}
        self.units = model_units(model)
        for u, m in enumerate(self.units):
            for p in m.parameters():
                unit_of.setdefault(id(p), u)
        n_units = len(self.units) + 1  # the last group: parameters outside every unit
        self._copies: List[List[Tuple[int, int, int]]] = [[] for _ in range(n_units)]
        for r, mem in enumerate(self.regions):
            if r in own:
                continue
            u = unit_of.get(id(self.params[mem[0]]), n_units - 1)
            src = self.pbuf.ptrs[self.plan.owner[r]] + self.plan.param_off[r]
            self._copies[u].append((self.params[mem[0]].data_ptr(), src, rbytes[r]))
        self._stream = torch.cuda.Stream(device=self.device)
        self._events: List[Optional[torch.cuda.Event]] = [None] * n_units
        self._hooks = [m.register_forward_pre_hook(self._make_hook(u)) for u, m in enumerate(self.units)]
        self.epoch = 0
        self.last_sumsq: Optional[torch.Tensor] = None
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        logger.info("fused FSDP: %d parameters in %d regions, %d owned by rank %d (%.1f MB of %.1f MB; "
                    "imbalance %.3f)", len(self.params), len(self.regions), len(self.owned), self.rank, self.plan.load[self.rank] / 2 ** 20,
                    sum(self.plan.load) / 2 ** 20, self.plan.imbalance())

    # ------------------------------------------------------------------ helpers
    @property
    def _flags(self) -> int:
        return self.pbuf.local_ptr + self.flag_off

    def _raise(self, row: int) -> None:
        self.C.fsdp_raise(self.pbuf.peer_base, self.flag_off, row, self.rank, self.world, self.epoch)

    def _wait(self, row: int) -> None:
        self.C.peer_flags_wait(self._flags + 4 * row * self.world, self.device.index, self.rank, self.world, 1,
                               self.epoch, self.wait_s)

    def _attach_grads(self) -> None:
        for p, v in zip(self.params, self._grad_views):
            g = p.grad
            if g is None:
                v.zero_()
            elif g.data_ptr() != v.data_ptr():
                v.copy_(g)
            p.grad = v

    def _make_hook(self, u: int):
        def hook(_module, _args):
            ev = self._events[u]
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
                self._events[u] = None
        return hook

    def wait_gathers(self) -> None:
        """Make the current stream wait for every pending parameter copy (checkpointing, eval)."""
        cur = torch.cuda.current_stream(self.device)
        for u, ev in enumerate(self._events):
            if ev is not None:
                cur.wait_event(ev)
                self._events[u] = None

    # ------------------------------------------------------------------ step
    def reduce(self) -> torch.Tensor:
        """Mean gradients of the owned parameters (in place) and the global squared norm."""
        self.wait_gathers()
        self.epoch += 1
        self._attach_grads()
        self._raise(self.READY)    # this rank's gradients are final
        self._wait(self.READY)     # ... and every peer's
        self.sumsq.zero_()
        self.C.fsdp_reduce(self.gbuf.peer_base, self.seg_off, self.seg_vec, self.total_vec, self.rank, self.world,
                           1.0 / self.world, self.sumsq)
        self._raise(self.REDUCED)  # this rank has read every peer's gradients
        dist.all_reduce(self.sumsq, group=self.group)
        for p in self.params:  # only owners step a parameter
            if id(p) not in self._own_ids:
                p.grad = None
        self.last_sumsq = self.sumsq
        return self.sumsq

    def after_optimizer_step(self) -> None:
        """Publish the owned parameters and start copying the others from their owners."""
        if self.epoch == 0:
            return
        cur = torch.cuda.current_stream(self.device)
        self._wait(self.REDUCED)   # no owner still reads this rank's gradients: they may be zeroed
        self._raise(self.PUBLISHED)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            self._wait(self.PUBLISHED)
            for u, copies in enumerate(self._copies):
                if not copies:
                    continue
                for dst, src, nb in copies:
                    self.C.peer_copy(dst, src, nb)
                ev = torch.cuda.Event()
                ev.record(self._stream)
                self._events[u] = ev
        # the tail group (parameters outside every unit, e.g. a tied head) is awaited at once
        if self._events[-1] is not None:
            cur.wait_event(self._events[-1])
            self._events[-1] = None
        for p, v in zip(self.params, self._grad_views):
            if p.grad is None:
                p.grad = v

    def close(self) -> None:
        for h in self._hooks:
            h.remove()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.gbuf.close()
        self.pbuf.close()
