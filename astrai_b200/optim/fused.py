"""Fused optimizers on the framework's kernels.

* :class:`FusedAdamW` - torch AdamW semantics (decoupled weight decay, bias
  correction) in ONE launch per parameter group over all tensors (pointer
  tables built once and cached), fp32 moments, bf16 or fp32 params.
* :class:`Muon` - torch.optim.Muon semantics (scripts/tools/train.py:58-72 in
  the reference uses it): Nesterov momentum, Frobenius normalisation, 5
  quintic Newton-Schulz iterations ``X <- aX + (bA + cA^2) X`` with
  ``A = X X^T`` (coefficients 3.4445, -4.7750, 2.0315; tall matrices are
  transposed first), decoupled weight decay and the ``original`` /
  ``match_rms_adamw`` learning-rate adjustment. All matrices of the same shape
  are orthogonalised together: each NS product is ONE batched tcgen05 GEMM
  over the whole stack (the reference runs 3 ATen matmuls per matrix per
  iteration, one matrix at a time).
* :class:`MuonMix` - the reference CLI's split (Muon on >=2-D weights whose
  name has none of norm/bias/embed/lm_head, AdamW(0.9, 0.95) elsewhere), with
  optional separate learning rates / weight decay for the two halves.
* :func:`clip_grad_norm_` - global L2 norm over all gradients in one launch;
  the clip coefficient stays on the device and is applied inside the update
  kernels, so a training step never waits for the host.

CPU parameters use the plain torch implementations (the CPU/gloo path).
"""

from __future__ import annotations

import os

import math
from typing import Dict, Iterable, List, Optional, Tuple

import torch
from torch.optim import Optimizer

from astrai_b200.ops._ext import native
from astrai_b200.utils.phase_timer import phase

NS_COEFFS = (3.4445, -4.7750, 2.0315)
CHUNK = 1 << 16


def _i64(vals: List[int], device) -> torch.Tensor:
    return torch.tensor(vals, dtype=torch.int64).to(device, non_blocking=False)


def _chunk_table(sizes: List[int], device) -> torch.Tensor:
    """[n_chunks] records (int tensor, int len, int64 start) packed as int32x4."""
    rows = []
    for t, n in enumerate(sizes):
        for s in range(0, n, CHUNK):
            ln = min(CHUNK, n - s)
            rows.append((t, ln, s & 0xFFFFFFFF, s >> 32))
    if not rows:
        return torch.zeros((0, 4), dtype=torch.int32, device=device)
    return torch.tensor(rows, dtype=torch.int64).to(torch.int32).to(device)


class GradClipState:
    """Device scalars shared by the clip and the optimizer kernels."""

    def __init__(self, device):
        self.acc = torch.zeros(1, device=device, dtype=torch.float32)
        self.coef = torch.ones(1, device=device, dtype=torch.float32)
        self.norm = torch.zeros(1, device=device, dtype=torch.float32)


_CLIP: Dict[torch.device, GradClipState] = {}


def clip_state(device) -> GradClipState:
    device = torch.device(device)
    if device not in _CLIP:
        _CLIP[device] = GradClipState(device)
    return _CLIP[device]


def clip_grad_norm_(params: Iterable[torch.Tensor], max_norm: Optional[float], apply_now: bool = False) -> torch.Tensor:
    """Global grad-norm; returns the norm as a device tensor.

    On CUDA the coefficient ``min(1, max_norm/(norm+1e-6))`` is left on the
    device and consumed by FusedAdamW/Muon in their next step (call
    ``apply_now=True`` to scale the gradients in place instead, e.g. for other
    optimizers). On CPU it behaves like ``torch.nn.utils.clip_grad_norm_``.
    """
    params = [p for p in params if p.grad is not None]
    if not params:
        return torch.zeros(())
    dev = params[0].grad.device
    if dev.type != "cuda" or any(p.grad.dtype != torch.bfloat16 for p in params):
        if max_norm is None:
            return torch.linalg.vector_norm(torch.stack([torch.linalg.vector_norm(p.grad.float()) for p in params]))
        return torch.nn.utils.clip_grad_norm_(params, max_norm)
    C = native()
    st = clip_state(dev)
    st.acc.zero_()
    sizes = [p.grad.numel() for p in params]
    key = ("clip", tuple(sizes))
    table = _TABLE_CACHE.get(key)
    if table is None:
        table = _chunk_table(sizes, dev)
        _TABLE_CACHE[key] = table
    gptr = _i64([p.grad.data_ptr() for p in params], dev)
    C.grad_sumsq(table, gptr, None, st.acc)
    C.clip_coef(st.acc, float(max_norm) if max_norm is not None else -1.0, st.coef, st.norm)
    if apply_now and max_norm is not None:
        for p in params:
            p.grad.mul_(st.coef.to(p.grad.dtype))
        st.coef.fill_(1.0)
    return st.norm[0]


_TABLE_CACHE: Dict[tuple, torch.Tensor] = {}


class FusedAdamW(Optimizer):
    def __init__(self, params, lr: float = 1e-3, betas: Tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01, use_clip_coef: bool = True):
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.use_clip_coef = use_clip_coef
        self._reset_clip = True  # the clip coefficient is consumed by one step
        self._tables: Dict[int, tuple] = {}

    def _group_tables(self, gi: int, params: List[torch.Tensor]):
        key = (gi, tuple(p.data_ptr() for p in params))
        cached = self._tables.get(gi)
        if cached is not None and cached[0] == key:
            return cached[1]
        dev = params[0].device
        for p in params:
            st = self.state[p]
            if "exp_avg" not in st:
                st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)
                st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32, memory_format=torch.contiguous_format)
                st["step"] = torch.zeros((), dtype=torch.float32)
        t = {
            "chunks": _chunk_table([p.numel() for p in params], dev),
            "p": _i64([p.data_ptr() for p in params], dev),
            "m": _i64([self.state[p]["exp_avg"].data_ptr() for p in params], dev),
            "v": _i64([self.state[p]["exp_avg_sq"].data_ptr() for p in params], dev),
        }
        self._tables[gi] = (key, t)
        return t

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            b1, b2 = group["betas"]
            lr, eps, wd = group["lr"], group["eps"], group["weight_decay"]
            if isinstance(lr, torch.Tensor):
                lr = float(lr)
            cuda_ok = params[0].is_cuda and all(p.is_contiguous() and p.dtype in (torch.bfloat16, torch.float32)
                                                 and p.grad.dtype == p.dtype and p.grad.is_contiguous()
                                                 for p in params)
            if not cuda_ok:
                self._step_reference(params, lr, b1, b2, eps, wd)
                continue
            fp32 = params[0].dtype == torch.float32
            if any((p.dtype == torch.float32) != fp32 for p in params):
                self._step_reference(params, lr, b1, b2, eps, wd)
                continue
            t = self._group_tables(gi, params)
            step = float(self.state[params[0]]["step"]) + 1.0
            for p in params:
                self.state[p]["step"].fill_(step)
            gptr = _i64([p.grad.data_ptr() for p in params], params[0].device)
            wdt = t.get("wd")
            if wdt is None or t.get("wd_val") != wd:
                t["wd"] = torch.full((len(params),), float(wd), dtype=torch.float32, device=params[0].device)
                t["wd_val"] = wd
            coef = clip_state(params[0].device).coef if self.use_clip_coef else None
            native().adamw_step(t["chunks"], t["p"], gptr, t["m"], t["v"], t["wd"], fp32, lr, b1, b2, eps,
                                1.0 - b1 ** step, 1.0 - b2 ** step, coef)
            if self._reset_clip and coef is not None:
                coef.fill_(1.0)
        return loss

    def _step_reference(self, params, lr, b1, b2, eps, wd):
        for p in params:
            st = self.state[p]
            if "exp_avg" not in st:
                st["exp_avg"] = torch.zeros_like(p, dtype=torch.float32)
                st["exp_avg_sq"] = torch.zeros_like(p, dtype=torch.float32)
                st["step"] = torch.zeros((), dtype=torch.float32)
            st["step"] += 1
            step = float(st["step"])
            g = p.grad.float()
            if p.is_cuda and self.use_clip_coef:
                g = g * clip_state(p.device).coef
            st["exp_avg"].mul_(b1).add_(g, alpha=1 - b1)
            st["exp_avg_sq"].mul_(b2).addcmul_(g, g, value=1 - b2)
            denom = (st["exp_avg_sq"] / (1 - b2 ** step)).sqrt_().add_(eps)
            pf = p.float().mul_(1 - lr * wd).addcdiv_(st["exp_avg"], denom, value=-lr / (1 - b1 ** step))
            p.copy_(pf.to(p.dtype))


def _adjust_lr(lr: float, mode: Optional[str], shape) -> float:
    A, B = shape[:2]
    if mode is None or mode == "original":
        return lr * math.sqrt(max(1.0, A / B))
    if mode == "match_rms_adamw":
        return lr * 0.2 * math.sqrt(max(A, B))
    return lr


def newton_schulz_reference(g: torch.Tensor, steps: int = 5, eps: float = 1e-7, coeffs=NS_COEFFS) -> torch.Tensor:
    """torch.optim.Muon's orthogonalisation (bf16), used as the CPU path and test oracle."""
    a, b, c = coeffs
    x = g.bfloat16()
    tall = g.size(0) > g.size(1)
    if tall:
        x = x.T
    x = x / x.norm().clamp(min=eps)
    for _ in range(steps):
        A = x @ x.T
        Bm = torch.addmm(A, A, A, beta=b, alpha=c)
        x = torch.addmm(x, Bm, x, beta=a)
    return x.T if tall else x


# ASTRAI_NS_SYM=0 computes every tile of the symmetric X X^T products
NS_SYM = os.environ.get("ASTRAI_NS_SYM", "1") == "1"


def newton_schulz_batched(X: torch.Tensor, steps: int = 5, coeffs=NS_COEFFS, work=None) -> torch.Tensor:
    """In-GPU batched NS on X [B, m, n] (m <= n, already normalised). Returns the result buffer."""
    C = native()
    a, b, c = coeffs
    Bn, m, n = X.shape
    if work is None:
        work = (torch.empty_like(X), torch.empty(Bn, m, m, device=X.device, dtype=X.dtype),
                torch.empty(Bn, m, m, device=X.device, dtype=X.dtype))
    Y, A, Bm = work
    cur, nxt = X, Y
    # A = X X^T and Bm = c A A + b A are symmetric: only the tiles on or above the diagonal are
    # computed (the tile walk enumerates just those), then the lower triangle is mirrored in
    sym = NS_SYM
    for _ in range(steps):
        C.gemm(cur, cur, A, None, 0, 0, 1.0, 0.0, 0, sym)           # A = X X^T
        C.gemm(A, A, Bm, A, 0, 0, c, b, 0, sym)                     # Bm = c A A + b A
        C.gemm(Bm, cur, nxt, cur, 0, 1, 1.0, a, 0)                  # X' = Bm X + a X
        cur, nxt = nxt, cur
    return cur


class Muon(Optimizer):
    """``shard=True`` (data parallelism with replicated parameters and all-reduced gradients):
    matrix i of every same-shape group is owned by rank ``i % world``; only the owner keeps its
    momentum and runs Newton-Schulz, and one kernel applies the update to every rank's copy over
    NVLink peer memory (the parameters are moved into a symmetric buffer on the first step).
    Parameters marked ``_ep_local`` (expert-parallel shards, different on every rank) stay local."""

    def __init__(self, params, lr: float = 1e-3, weight_decay: float = 0.1, momentum: float = 0.95,
                 nesterov: bool = True, ns_coefficients=NS_COEFFS, eps: float = 1e-7, ns_steps: int = 5,
                 adjust_lr_fn: Optional[str] = None, use_clip_coef: bool = True, shard: bool = False,
                 process_group=None, wait_s: float = 60.0):
        super().__init__(params, dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                                      ns_coefficients=tuple(ns_coefficients), eps=eps, ns_steps=ns_steps,
                                      adjust_lr_fn=adjust_lr_fn))
        for g in self.param_groups:
            for p in g["params"]:
                if p.dim() != 2:
                    raise ValueError("Muon only supports 2-D parameters")
        self.use_clip_coef = use_clip_coef
        self._reset_clip = True
        self._work: Dict[tuple, dict] = {}
        self.shard, self.process_group, self.wait_s = shard, process_group, wait_s
        self._arena = None
        self._epoch = 0

    @property
    def sharded(self) -> bool:
        import torch.distributed as dist

        return bool(self.shard and dist.is_available() and dist.is_initialized()
                    and dist.get_world_size(self.process_group) > 1)

    def _buf(self, p):
        st = self.state[p]
        if "momentum_buffer" not in st:
            st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32 if p.is_cuda else p.dtype)
        return st["momentum_buffer"]

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        if self.sharded:
            self._step_sharded()
            return loss
        for gi, group in enumerate(self.param_groups):
            params = [p for p in group["params"] if p.grad is not None]
            if not params:
                continue
            if not params[0].is_cuda or any(p.dtype != torch.bfloat16 for p in params):
                self._step_reference(params, group)
                continue
            by_shape: Dict[tuple, List[torch.Tensor]] = {}
            for p in params:
                by_shape.setdefault(tuple(p.shape), []).append(p)
            for shape, ps in by_shape.items():
                with phase("muon_newton_schulz"):
                    self._step_batched(gi, shape, ps, group)
            if self._reset_clip and self.use_clip_coef:
                clip_state(params[0].device).coef.fill_(1.0)
        return loss

    # ------------------------------------------------------------------ owner-sharded step
    def _shared_groups(self):
        """[(gi, shape, params)] of the replicated matrices, in the same order on every rank."""
        out = []
        for gi, group in enumerate(self.param_groups):
            by_shape: Dict[tuple, List[torch.Tensor]] = {}
            for p in group["params"]:
                if not getattr(p, "_ep_local", False):
                    by_shape.setdefault(tuple(p.shape), []).append(p)
            out += [(gi, shape, ps) for shape, ps in by_shape.items()]
        return out

    def _step_sharded(self):
        import torch.distributed as dist

        from astrai_b200.parallel.symm import ParamArena

        groups = self._shared_groups()
        shared = [p for _, _, ps in groups for p in ps]
        if shared and (self._arena is None or not all(self._arena.holds(p) for p in shared)):
            if self._arena is not None:  # parameters were re-packed elsewhere: rebuild on every rank
                dist.barrier(group=self.process_group)
            self._arena = ParamArena(shared, self.process_group)
            self._work = {k: v for k, v in self._work.items() if k[0] != "own"}
        if len(groups) > ParamArena.FLAG_ROWS:
            raise RuntimeError(f"sharded Muon supports at most {ParamArena.FLAG_ROWS} shape groups")
        C = native()
        a = self._arena
        W, r = (a.world, a.rank) if a is not None else (1, 0)
        self._epoch += 1
        dev = None
        for slot, (gi, shape, ps) in enumerate(groups):
            group = self.param_groups[gi]
            own = [p for i, p in enumerate(ps) if i % W == r]
            if any(p.grad is None for p in own):
                raise RuntimeError("sharded Muon: an owned parameter has no gradient")
            R, Cc = shape
            lr = float(group["lr"])
            adj = _adjust_lr(lr, group["adjust_lr_fn"], shape)
            dev = ps[0].device
            if own:
                chunks = _ns_chunks(own)
                for ci, chunk in enumerate(chunks):
                    with phase("muon_newton_schulz"):
                        t, out, tall = self._orthogonalize(("own", gi, shape, ci), chunk, group)
                    # only the group's last launch raises its flag on the peers (slot -1: no flag); the
                    # earlier launches' stores precede it in stream order
                    with phase("muon_apply_peers"):
                        C.muon_apply_peers(t["pptr"], t["poff"], a.buf.peer_base, out, len(chunk), R, Cc, tall,
                                           1.0 - lr * group["weight_decay"], adj, r, W, a.flag_off,
                                           slot if ci == len(chunks) - 1 else -1, self._epoch, a.done)
            else:  # nothing owned in this group: only raise its flag on the peers
                C.muon_apply_peers(None, None, a.buf.peer_base, None, 0, R, Cc, False, 1.0, 0.0, r, W, a.flag_off,
                                   slot, self._epoch, a.done)
        # expert-parallel shards: every rank updates its own
        for gi, group in enumerate(self.param_groups):
            local = [p for p in group["params"] if getattr(p, "_ep_local", False) and p.grad is not None]
            by_shape: Dict[tuple, List[torch.Tensor]] = {}
            for p in local:
                by_shape.setdefault(tuple(p.shape), []).append(p)
            for shape, ps in by_shape.items():
                self._step_batched(gi, shape, ps, group)
        if groups:
            with phase("muon_flag_wait"):
                C.peer_flags_wait(a.flags_addr, dev.index, r, W, len(groups), self._epoch, self.wait_s)
        if self._reset_clip and self.use_clip_coef and dev is not None:
            clip_state(dev).coef.fill_(1.0)

    def _scratch(self, shape, Bn, dev):
        """Newton-Schulz scratch for ``Bn`` matrices of ``shape``, shared by every group and chunk of that
        shape and size (momentum lives in the optimizer state; nothing here outlives one call)."""
        key = ("scratch", shape, Bn)
        s = self._work.get(key)
        if s is None:
            R, Cc = shape
            m, n = (Cc, R) if R > Cc else (R, Cc)
            s = {
                "U": torch.empty(Bn, R, Cc, device=dev, dtype=torch.bfloat16),
                "X": torch.empty(Bn, m, n, device=dev, dtype=torch.bfloat16),
                "Y": torch.empty(Bn, m, n, device=dev, dtype=torch.bfloat16),
                "A": torch.empty(Bn, m, m, device=dev, dtype=torch.bfloat16),
                "Bm": torch.empty(Bn, m, m, device=dev, dtype=torch.bfloat16),
                "sumsq": torch.zeros(Bn, device=dev, dtype=torch.float32),
            }
            self._work[key] = s
        return s

    def _orthogonalize(self, key, ps, group):
        """Momentum + Frobenius normalisation + Newton-Schulz of the same-shape matrices ``ps`` (one
        chunk, see ``_ns_chunks``); returns the chunk's pointer tables, the update and its layout."""
        C = native()
        dev = ps[0].device
        R, Cc = ps[0].shape
        tall = R > Cc
        s = self._scratch((R, Cc), len(ps), dev)
        ident = tuple(p.data_ptr() for p in ps)
        t = self._work.get(key)
        if t is None or t["ident"] != ident:
            t = {"ident": ident, "pptr": _i64([p.data_ptr() for p in ps], dev),
                 "bptr": _i64([self._buf(p).data_ptr() for p in ps], dev)}
            if self._arena is not None and all(self._arena.holds(p) for p in ps):
                t["poff"] = _i64([self._arena.offset[id(p)] for p in ps], dev)
            self._work[key] = t
        gptr = _i64([p.grad.data_ptr() for p in ps], dev)
        s["sumsq"].zero_()
        coef = clip_state(dev).coef if self.use_clip_coef else None
        C.muon_momentum(gptr, t["bptr"], True, s["U"], group["momentum"], group["nesterov"], coef, s["sumsq"])
        C.muon_normalize(s["U"], s["X"], tall, s["sumsq"], group["eps"])
        out = newton_schulz_batched(s["X"], group["ns_steps"], group["ns_coefficients"], (s["Y"], s["A"], s["Bm"]))
        return t, out, tall

    def _step_batched(self, gi, shape, ps, group):
        R, Cc = shape
        lr = float(group["lr"])
        adj = _adjust_lr(lr, group["adjust_lr_fn"], shape)
        for ci, chunk in enumerate(_ns_chunks(ps)):
            t, out, tall = self._orthogonalize((gi, shape, ci), chunk, group)
            native().muon_apply(t["pptr"], False, out, R, Cc, tall, 1.0 - lr * group["weight_decay"], adj)

    def _step_reference(self, params, group):
        mu = group["momentum"]
        for p in params:
            buf = self._buf(p)
            g = p.grad
            if p.is_cuda and self.use_clip_coef:
                g = g * clip_state(p.device).coef.to(g.dtype)
            buf.lerp_(g.to(buf.dtype), 1 - mu)
            upd = g.lerp(buf.to(g.dtype), mu) if group["nesterov"] else buf
            upd = newton_schulz_reference(upd, group["ns_steps"], group["eps"], group["ns_coefficients"])
            lr = float(group["lr"])
            p.mul_(1 - lr * group["weight_decay"])
            p.add_(upd.to(p.dtype), alpha=-_adjust_lr(lr, group["adjust_lr_fn"], p.shape))


# bf16 bytes of the matrices one batched Newton-Schulz chain handles at a time: the scratch (update,
# two iterates, two Gram matrices) is about 5x this, so a model with thousands of same-shape matrices
# (MoE experts) keeps a bounded workspace instead of one sized for every matrix of the shape.
_NS_CHUNK_BYTES = int(os.environ.get("ASTRAI_NS_CHUNK_BYTES", str(1 << 30)))


def _ns_chunks(ps):
    """``ps`` split into near-equal chunks of at most ``_NS_CHUNK_BYTES`` (at least one matrix each)."""
    R, Cc = ps[0].shape
    n = max(1, -(-len(ps) * R * Cc * 2 // max(1, _NS_CHUNK_BYTES)))
    per = -(-len(ps) // n)
    return [ps[i:i + per] for i in range(0, len(ps), per)]


def is_muon_param(name: str, p: torch.Tensor) -> bool:
    """The reference CLI's rule (scripts/tools/train.py:44-54)."""
    return p.dim() >= 2 and not any(s in name for s in ("norm", "bias", "embed", "lm_head"))


class MuonMix(Optimizer):
    """Muon on hidden matrices + AdamW(0.9, 0.95) on the rest, one object."""

    def __init__(self, model: torch.nn.Module, lr: float = 3e-4, weight_decay: float = 0.1, momentum: float = 0.95,
                 nesterov: bool = True, ns_steps: int = 5, adjust_lr_fn: Optional[str] = "match_rms_adamw",
                 adamw_lr: Optional[float] = None, adamw_weight_decay: float = 0.0,
                 adamw_betas: Tuple[float, float] = (0.9, 0.95), shard_muon: bool = False, process_group=None):
        params = [p for p in model.parameters() if p.requires_grad]
        super().__init__(params, dict(lr=lr))
        seen = set()
        mat, other = [], []
        for name, p in model.named_parameters():
            if not p.requires_grad or id(p) in seen:
                continue
            seen.add(id(p))
            (mat if is_muon_param(name, p) else other).append(p)
        self.muon = Muon(mat, lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                         ns_steps=ns_steps, adjust_lr_fn=adjust_lr_fn, shard=shard_muon,
                         process_group=process_group) if mat else None
        self.adamw = FusedAdamW([{"params": other, "weight_decay": adamw_weight_decay}],
                                lr=adamw_lr if adamw_lr is not None else lr, betas=adamw_betas) if other else None
        self.param_groups = [*(self.muon.param_groups if self.muon else []),
                             *(self.adamw.param_groups if self.adamw else [])]
        for o in (self.muon, self.adamw):
            if o is not None:
                o._reset_clip = False
        self._device = params[0].device if params else None

    @torch.no_grad()
    def step(self, closure=None):
        if self.muon:
            self.muon.step()
        if self.adamw:
            with phase("adamw"):
                self.adamw.step()
        if self._device is not None and self._device.type == "cuda":
            clip_state(self._device).coef.fill_(1.0)

    def zero_grad(self, set_to_none: bool = True):
        if self.muon:
            self.muon.zero_grad(set_to_none)
        if self.adamw:
            self.adamw.zero_grad(set_to_none)

    @property
    def sharded(self) -> bool:
        """True when every rank holds different optimizer state (save one file per rank)."""
        return bool(self.muon is not None and self.muon.sharded)

    def state_dict(self):
        return {"muon": self.muon.state_dict() if self.muon else {},
                "adamw": self.adamw.state_dict() if self.adamw else {}}

    def load_state_dict(self, state_dict):
        if self.muon and state_dict.get("muon"):
            self.muon.load_state_dict(state_dict["muon"])
        if self.adamw and state_dict.get("adamw"):
            self.adamw.load_state_dict(state_dict["adamw"])
        self.param_groups = [*(self.muon.param_groups if self.muon else []),
                             *(self.adamw.param_groups if self.adamw else [])]
