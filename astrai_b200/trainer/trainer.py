"""Trainer (parity: astrai/trainer/trainer.py:15-113).

``Trainer(train_config, callbacks).train(param_path, resume)`` spawns the
ranks (``spawn_parallel_fn``), builds the context and runs the epoch / batch
loop with gradient accumulation, callbacks, optimizer / scheduler steps on
sync micro-steps, and ``on_error`` (checkpoint + metric flush) on failure.

Unlike the reference loop, the per-micro-batch ``loss.item()`` host sync is
gone: the loss stays on the device (``context.loss`` reads it lazily, once
per optimizer step by the progress bar / metrics), so the GPU queue never
drains between micro-batches.
"""

from __future__ import annotations

import logging
from typing import List, Optional

import torch

from astrai_b200.config.train_config import TrainConfig
from astrai_b200.parallel.setup import spawn_parallel_fn
from astrai_b200.trainer.train_callback import CallbackFactory, TrainCallback, nvtx_range
from astrai_b200.trainer.graph_step import GraphedMicroStep
from astrai_b200.trainer.train_context import TrainContext, TrainContextBuilder

logger = logging.getLogger(__name__)


def _batch_tokens(batch) -> int:
    """Token positions processed by one micro-batch on this rank (the largest id tensor of the batch dict)."""
    if not isinstance(batch, dict):
        return 0
    n = [v.numel() for v in batch.values() if hasattr(v, "dtype") and not v.is_floating_point() and v.dim() >= 2]
    return max(n, default=0)


class Trainer:
    def __init__(self, train_config: TrainConfig, callbacks: Optional[List[TrainCallback]] = None):
        self.train_config = train_config
        self.callbacks = self._default_callbacks() + list(callbacks or [])
        self.last_context: Optional[TrainContext] = None

    def _default_callbacks(self) -> List[TrainCallback]:
        c = self.train_config
        cbs = [
            CallbackFactory.create("gradient_checkpointing", modules=c.gradient_checkpointing_modules),
            CallbackFactory.create("checkpoint", c.ckpt_dir, c.ckpt_interval),
            CallbackFactory.create("metric", log_dir=c.log_dir, save_interval=c.ckpt_interval, metrics=c.metrics,
                                   val_step=c.val_step),
            CallbackFactory.create("progress_bar", c.n_epoch),
            CallbackFactory.create("gradient_clipping", c.max_grad_norm),
        ]
        if c.profile_dir:
            cbs.append(CallbackFactory.create("profiler", profile_dir=c.profile_dir))
        if c.nprocs > 1:
            cbs.append(CallbackFactory.create("health"))
        return cbs

    def _call(self, name: str, ctx: TrainContext) -> None:
        for cb in self.callbacks:
            fn = getattr(cb, name, None)
            if fn is not None:
                fn(ctx)

    def _graph_runner(self, ctx: TrainContext):
        """The CUDA-graph micro-step when ``cuda_graph`` is set and this run can use it."""
        c, ex, st = ctx.config, ctx.executor, ctx.strategy
        if not getattr(c, "cuda_graph", False):
            return None
        why = None
        if not getattr(st, "cuda_graph_safe", False) or getattr(st, "_rollout_runner", None) is not None:
            why = f"strategy {type(st).__name__} is not graph-safe"
        elif not getattr(ex, "cuda_graph_safe", False):
            why = f"executor {type(ex).__name__} is not graph-safe"
        elif torch.device(ctx.strategy.device).type != "cuda":
            why = "not on a CUDA device"
        if why is not None:
            logger.warning("cuda_graph requested but %s: running eagerly", why)
            return None
        return GraphedMicroStep(st, ex.unwrap(ctx.model), torch.device(st.device), scale=1.0 / ex.grad_accum_steps,
                                eager_calls=ex.grad_accum_steps)

    def _trainer_loop(self, param_path: Optional[str] = None, resume: bool = False) -> None:
        ctx = TrainContextBuilder(self.train_config).with_param_path(param_path, resume=resume).build()
        self.last_context = ctx
        ex = ctx.executor
        graph = self._graph_runner(ctx)
        ctx.kwargs["graph_step"] = graph
        per_micro = ctx.config.batch_per_device * ctx.world_size
        self._call("on_train_begin", ctx)
        try:
            ctx.model.train()
            for epoch in range(ctx.epoch, ctx.config.n_epoch):
                ctx.epoch = epoch
                self._call("on_epoch_begin", ctx)
                for batch in ctx.dataloader:
                    with ex.accumulate(ctx.model):
                        self._call("on_batch_begin", ctx)
                        if graph is not None:
                            with nvtx_range("forward_backward"):
                                ctx.loss = graph(batch)
                            if ex.sync_gradients and ex.use_distributed:
                                ex._reduce_gradients()
                        else:
                            with nvtx_range("forward"):
                                loss = ctx.strategy(batch)
                            ctx.loss = loss.detach()
                            with nvtx_range("backward"):
                                ex.backward(loss / ex.grad_accum_steps)
                        ctx.consumed_samples += per_micro
                        ctx.kwargs["tokens"] = ctx.kwargs.get("tokens", 0) + _batch_tokens(batch) * ctx.world_size
                        self._call("on_batch_end", ctx)
                        if ex.sync_gradients:
                            self._call("on_optimizer_step", ctx)
                            with nvtx_range("optimizer"):
                                ctx.optimizer.step()
                            ctx.strategy.on_optimizer_step()
                            # the graph accumulates into gradients that stay allocated
                            ctx.optimizer.zero_grad(set_to_none=graph is None)
                            if ctx.scheduler:
                                ctx.scheduler.step()
                self._call("on_epoch_end", ctx)
        except Exception as e:
            logger.error("Training failed: %s", e, exc_info=True)
            self._call("on_error", ctx)
            raise
        finally:
            self._call("on_train_end", ctx)

    def train(self, param_path: Optional[str] = None, resume: bool = False) -> None:
        c = self.train_config
        spawn_parallel_fn(self._trainer_loop, backend=c.backend, world_size=c.nprocs, master_addr=c.master_addr,
                          master_port=c.master_port, device_type=c.device_type, start_method=c.start_method,
                          param_path=param_path, resume=resume)
