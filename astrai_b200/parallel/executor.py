"""Training executors: gradient accumulation + data / sharded parallelism.

API parity with the reference (astrai/parallel/executor.py): ``GradientState``,
``AccumOptimizer``/``AccumScheduler`` (step only on sync micro-steps),
``BaseExecutor.prepare(model_fn, optimizer_fn, scheduler_fn, before_wrap)``,
``accumulate(model)``, ``backward(loss)``, ``unwrap_model(model)`` (full state
dict), ``checkpoint_context(model)`` (barrier, rank-0 state dict, barrier),
``clip_grad_norm(model, max_norm)``, ``sync_gradients``, ``grad_accum_steps``;
registered as ``none``, ``ddp``, ``fsdp``, ``fsdp2``.

Design differences (B200-first):
* ``ddp`` keeps a replica per GPU and exchanges gradients ONCE per optimizer
  step, after the last micro-batch (no per-micro-step hooks), through
  :mod:`astrai_b200.parallel.comm` - NCCL all-reduce (``comm_backend="nccl"``)
  or the framework's own NVLink peer-memory all-reduce kernel that also
  produces the squared gradient norm (``comm_backend="fused"``).
* ``fsdp`` / ``fsdp2`` shard parameters with torch's ``fully_shard`` per
  decoder block (as the reference's FSDP2 executor does).
* Gradient clipping uses the fused global-norm kernel; the coefficient is
  applied inside the optimizer kernels.
"""

from __future__ import annotations

import contextlib
import logging
from contextlib import contextmanager
from typing import Any, Callable, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from astrai_b200.factory import Registry
from astrai_b200.parallel.setup import get_rank, get_world_size

logger = logging.getLogger(__name__)


class GradientState:
    def __init__(self, grad_accum_steps: int = 1):
        self.num_steps = max(int(grad_accum_steps), 1)
        self._step = 0
        self._sync_gradients = True

    @property
    def sync_gradients(self) -> bool:
        return self._sync_gradients

    def _do_sync(self) -> None:
        self._step += 1
        self._sync_gradients = self._step % self.num_steps == 0


class AccumOptimizer:
    def __init__(self, optimizer, gradient_state: GradientState, on_step: Optional[Callable[[], None]] = None):
        self.optimizer = optimizer
        self.gradient_state = gradient_state
        self.on_step = on_step  # the executor's work after an optimizer step (publishing sharded parameters)

    def step(self, closure=None):
        if self.gradient_state.sync_gradients:
            self.optimizer.step(closure) if closure is not None else self.optimizer.step()
            if self.on_step is not None:
                self.on_step()

    def zero_grad(self, set_to_none: bool = True):
        if self.gradient_state.sync_gradients:
            self.optimizer.zero_grad(set_to_none)

    @property
    def param_groups(self):
        return self.optimizer.param_groups

    def state_dict(self):
        return self.optimizer.state_dict()

    def load_state_dict(self, d):
        self.optimizer.load_state_dict(d)


class AccumScheduler:
    def __init__(self, scheduler, gradient_state: GradientState):
        self.scheduler = scheduler
        self.gradient_state = gradient_state

    def step(self):
        if self.gradient_state.sync_gradients:
            self.scheduler.step()

    def state_dict(self):
        return self.scheduler.state_dict()

    def load_state_dict(self, d):
        self.scheduler.load_state_dict(d)

    def get_last_lr(self):
        return self.scheduler.get_last_lr()


class BaseExecutor:
    def __init__(self, grad_accum_steps: int = 1):
        self.gradient_state = GradientState(grad_accum_steps)
        self.last_grad_norm: Optional[torch.Tensor] = None

    # ------------------------------------------------------------------ setup
    def prepare(self, model_fn: Callable[[], nn.Module], optimizer_fn=None, scheduler_fn=None,
                before_wrap: Optional[Callable[[nn.Module], nn.Module]] = None) -> Tuple[nn.Module, Any, Any]:
        model = model_fn()
        if before_wrap is not None:
            model = before_wrap(model)
        model = self.wrap(model)
        optimizer = scheduler = None
        if optimizer_fn is not None:
            optimizer = optimizer_fn(self.unwrap(model))
            if scheduler_fn is not None:
                scheduler = scheduler_fn(optimizer)
            optimizer = AccumOptimizer(optimizer, self.gradient_state, self.after_optimizer_step)
            if scheduler is not None:
                scheduler = AccumScheduler(scheduler, self.gradient_state)
        return model, optimizer, scheduler

    def wrap(self, model: nn.Module) -> nn.Module:
        return model

    def unwrap(self, model: nn.Module) -> nn.Module:
        return model

    # ------------------------------------------------------------------ accumulation
    def _no_sync(self, model: nn.Module):
        return contextlib.nullcontext()

    @contextmanager
    def accumulate(self, model: nn.Module):
        self.gradient_state._do_sync()
        if not self.gradient_state.sync_gradients:
            with self._no_sync(model):
                yield
        else:
            yield

    def backward(self, loss: torch.Tensor) -> None:
        loss.backward()
        if self.sync_gradients and self.use_distributed:
            self._reduce_gradients()

    # explicit-loop helpers (used by bench / fused training loops)
    @contextmanager
    def micro_step(self, model: nn.Module, is_last: bool):
        if is_last:
            yield
        else:
            with self._no_sync(model):
                yield

    def finish_step(self, model: nn.Module) -> None:
        if self.use_distributed:
            self._reduce_gradients(model)

    def after_optimizer_step(self) -> None:
        """Called after every optimizer step (explicit loops call it themselves)."""

    def _reduce_gradients(self, model: Optional[nn.Module] = None) -> None:
        pass

    # ------------------------------------------------------------------ state
    def unwrap_model(self, model: nn.Module):
        return self.unwrap(model).state_dict()

    @contextmanager
    def checkpoint_context(self, model: nn.Module):
        if self.use_distributed:
            dist.barrier()
        sd = self._gather_state_dict(model)
        yield sd
        if self.use_distributed:
            dist.barrier()

    def _gather_state_dict(self, model: nn.Module):
        sd = self.unwrap_model(model)
        if self.use_distributed and get_rank() != 0:
            return None
        return sd

    @property
    def use_distributed(self) -> bool:
        return get_world_size() > 1

    @property
    def sync_gradients(self) -> bool:
        return self.gradient_state.sync_gradients

    @property
    def grad_accum_steps(self) -> int:
        return self.gradient_state.num_steps

    def clip_grad_norm(self, model: nn.Module, max_norm: Optional[float], as_tensor: bool = False):
        from astrai_b200.optim.fused import clip_grad_norm_

        norm = clip_grad_norm_(self.unwrap(model).parameters(), max_norm)
        self.last_grad_norm = norm
        if as_tensor:
            return norm
        return float(norm) if isinstance(norm, torch.Tensor) else norm


class ExecutorFactory(Registry[BaseExecutor]):
    pass


@ExecutorFactory.register("none")
class NoneExecutor(BaseExecutor):
    cuda_graph_safe = True  # nothing happens between backward and the optimizer step


@ExecutorFactory.register("ddp")
class DDPExecutor(BaseExecutor):
    """Replicated parameters, one gradient all-reduce (mean) per optimizer step."""

    cuda_graph_safe = True  # the all-reduce runs after the last micro-step, outside any graph

    def __init__(self, grad_accum_steps: int = 1, comm_backend: str = "nccl", bucket_cap_mb: int = 256,
                 broadcast_params: bool = True, expert_parallel: bool = False, **_ignored):
        super().__init__(grad_accum_steps)
        self.comm_backend = comm_backend
        self.bucket_cap_mb = bucket_cap_mb
        self.broadcast_params = broadcast_params
        self.expert_parallel = expert_parallel
        self._model: Optional[nn.Module] = None
        self._reducer = None

    def wrap(self, model: nn.Module) -> nn.Module:
        """Replicate (broadcast from rank 0); with ``expert_parallel`` every MoE
        layer then keeps only its share of the routed experts (EP over the
        data-parallel group, experts exchanged through NVLink peer memory)."""
        self._model = model
        if self.use_distributed and self.broadcast_params:
            with torch.no_grad():
                for t in list(model.parameters()) + list(model.buffers()):
                    if not getattr(t, "_ep_local", False):  # expert shards differ per rank by design
                        dist.broadcast(t.data, src=0)
        if self.use_distributed and self.expert_parallel:
            for m in model.modules():
                if hasattr(m, "shard_experts"):
                    m.shard_experts()
        return model

    def _reduce_gradients(self, model: Optional[nn.Module] = None) -> None:
        from astrai_b200.parallel.comm import GradReducer

        m = model if model is not None else self._model
        if self._reducer is None:
            self._reducer = GradReducer(m, backend=self.comm_backend, bucket_cap_mb=self.bucket_cap_mb)
        self._reducer.reduce()

    def clip_grad_norm(self, model: nn.Module, max_norm: Optional[float], as_tensor: bool = False):
        r = self._reducer
        if r is None or r.last_sumsq is None:
            return super().clip_grad_norm(model, max_norm, as_tensor)
        # the fused all-reduce already produced the global squared norm
        from astrai_b200.ops._ext import native
        from astrai_b200.optim.fused import clip_state

        st = clip_state(r.last_sumsq.device)
        native().clip_coef(r.last_sumsq, float(max_norm) if max_norm is not None else -1.0, st.coef, st.norm)
        r.last_sumsq = None
        norm = st.norm[0]
        self.last_grad_norm = norm
        return norm if as_tensor else float(norm)


@ExecutorFactory.register("fsdp2")
class FSDP2Executor(BaseExecutor):
    """Sharded data parallelism.

    ``comm_backend="nccl"`` (default): torch ``fully_shard`` on every child module, as the reference
    does (astrai/parallel/executor.py:316-407). ``comm_backend="fused"`` (CUDA, bf16, world > 1):
    whole-tensor owners over NVLink peer memory (:mod:`astrai_b200.parallel.fsdp`): gradients reduced
    to their owner in one kernel per step, the optimizer state and update sharded, parameters copied
    from their owners by the copy engines after each optimizer step."""

    def __init__(self, grad_accum_steps: int = 1, mesh=None, mp_policy=None, reshard_after_forward: bool = True,
                 comm_backend: str = "nccl", wait_s: float = 60.0, **_ignored):
        super().__init__(grad_accum_steps)
        self._kw = {k: v for k, v in dict(mesh=mesh, mp_policy=mp_policy,
                                          reshard_after_forward=reshard_after_forward).items() if v is not None}
        self.comm_backend = comm_backend
        self.wait_s = wait_s
        self._fused = None

    @property
    def cuda_graph_safe(self) -> bool:
        # torch FSDP2 and the fused backend both issue collectives or copies inside the micro-step
        return False

    def wrap(self, model: nn.Module) -> nn.Module:
        if not self.use_distributed:
            return model
        if self.comm_backend == "fused":
            from astrai_b200.parallel.fsdp import FusedFSDP

            self._fused = FusedFSDP(model, wait_s=self.wait_s)
            return model
        from torch.distributed.fsdp import fully_shard

        from astrai_b200.ops.gemm import set_packing

        set_packing(False)  # fully_shard owns the parameter storage from here on
        for child in model.children():
            if isinstance(child, nn.ModuleList):
                for sub in child:
                    fully_shard(sub, **self._kw)
            elif any(True for _ in child.parameters()):
                fully_shard(child, **self._kw)
        return model

    @contextmanager
    def _no_sync(self, model: nn.Module):
        if self._fused is not None:  # gradients accumulate locally until the step's reduction anyway
            yield
            return
        from torch.distributed.fsdp import FSDPModule

        mods = [m for m in model.modules() if isinstance(m, FSDPModule)]
        for m in mods:
            m.set_requires_gradient_sync(False, recurse=True)
        try:
            yield
        finally:
            for m in mods:
                m.set_requires_gradient_sync(True, recurse=True)

    def backward(self, loss: torch.Tensor) -> None:
        loss.backward()
        if self._fused is not None and self.sync_gradients:
            self._fused.reduce()

    def finish_step(self, model: nn.Module) -> None:
        if self._fused is not None:
            self._fused.reduce()

    def after_optimizer_step(self) -> None:
        if self._fused is not None:
            self._fused.after_optimizer_step()

    def clip_grad_norm(self, model: nn.Module, max_norm: Optional[float], as_tensor: bool = False):
        if not self.use_distributed:
            return super().clip_grad_norm(model, max_norm, as_tensor)
        if self._fused is not None and self._fused.last_sumsq is not None:
            from astrai_b200.ops._ext import native
            from astrai_b200.optim.fused import clip_state

            sumsq = self._fused.last_sumsq
            st = clip_state(sumsq.device)
            native().clip_coef(sumsq, float(max_norm) if max_norm is not None else -1.0, st.coef, st.norm)
            self._fused.last_sumsq = None
            norm = st.norm[0]
            self.last_grad_norm = norm
            return norm if as_tensor else float(norm)
        norm = torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm if max_norm is not None else float("inf"))
        self.last_grad_norm = norm
        return norm if as_tensor else float(norm)

    def unwrap_model(self, model: nn.Module):
        if not self.use_distributed:
            return model.state_dict()
        if self._fused is not None:
            self._fused.wait_gathers()
            sd = {k: v for k, v in model.state_dict().items()}
            return sd if get_rank() == 0 else None
        from torch.distributed.tensor import DTensor

        sd = model.state_dict()
        out = {k: (v.full_tensor() if isinstance(v, DTensor) else v) for k, v in sd.items()}
        return out if get_rank() == 0 else None


ExecutorFactory.alias("fsdp", "fsdp2")
