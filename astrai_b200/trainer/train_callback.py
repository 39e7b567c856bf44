"""Trainer callbacks (parity: astrai/trainer/train_callback.py).

Hooks: on_train_begin/end, on_epoch_begin/end, on_batch_begin/end,
on_optimizer_step, on_error. Registered callbacks:

* ``gradient_checkpointing`` - wraps ``forward`` of the listed module types
  with ``torch.utils.checkpoint`` (non-reentrant);
* ``checkpoint`` - saves ``ckpt_dir/epoch_{e}_step_{s}/`` every ``interval``
  optimizer steps, at the end and on error (model, meta.json with the train
  config, optimizer.pt, scheduler.pt);
* ``metric`` - JSONL metrics (loss, lr, grad_norm, val_loss) flushed to
  ``log_dir/epoch_{e}_step_{s}_metric.jsonl``; periodic validation with an
  all-reduced mean loss;
* ``progress_bar`` - rank-0 tqdm;
* ``gradient_clipping`` - global-norm clipping before the optimizer step.

Host/device synchronisation happens at most once per optimizer step (the
loss / grad-norm scalars are read when logged), not once per micro-batch.
"""

from __future__ import annotations

import json
import os
import sys
import time
from contextlib import contextmanager
from pathlib import Path
from typing import IO, Callable, List, Optional, Protocol, runtime_checkable

import torch
import torch.distributed as dist
import torch.nn as nn
from torch.utils.checkpoint import checkpoint as torch_checkpoint

from astrai_b200.factory import Registry
from astrai_b200.parallel.setup import get_current_device, get_rank, only_on_rank
from astrai_b200.serialization import Checkpoint


@runtime_checkable
class TrainCallback(Protocol):
    def on_train_begin(self, context): ...

    def on_train_end(self, context): ...

    def on_epoch_begin(self, context): ...

    def on_epoch_end(self, context): ...

    def on_batch_begin(self, context): ...

    def on_batch_end(self, context): ...

    def on_optimizer_step(self, context): ...

    def on_error(self, context): ...


class CallbackFactory(Registry):
    pass


@CallbackFactory.register("gradient_checkpointing")
class GradientCheckpointingCallback:
    def __init__(self, modules: Optional[List] = None):
        self.modules = tuple(modules or ())

    def _enable(self, m: nn.Module):
        if self.modules and isinstance(m, self.modules) and not hasattr(m, "_astrai_orig_forward"):
            m._astrai_orig_forward = m.forward

            def fwd(*a, __m=m, **k):
                if torch.is_grad_enabled():
                    return torch_checkpoint(__m._astrai_orig_forward, *a, use_reentrant=False, **k)
                return __m._astrai_orig_forward(*a, **k)

            m.forward = fwd

    def _disable(self, m: nn.Module):
        if hasattr(m, "_astrai_orig_forward"):
            m.forward = m._astrai_orig_forward
            del m._astrai_orig_forward

    def on_train_begin(self, context):
        if self.modules:
            context.model.apply(self._enable)

    def on_train_end(self, context):
        context.model.apply(self._disable)


@CallbackFactory.register("checkpoint")
class CheckpointCallback:
    extra_keys = ("optimizer", "scheduler")

    def __init__(self, save_dir: str, interval: int, weight_only: bool = False,
                 save_extra_fn: Optional[Callable] = None):
        self.save_dir = save_dir
        self.interval = interval
        self.weight_only = weight_only
        self.save_extra_fn = save_extra_fn or CheckpointCallback.save_extra
        self.last_ckpt_step = None

    def on_train_begin(self, context):
        self.last_ckpt_step = context.optimizer_step

    def _save(self, context):
        self.last_ckpt_step = context.optimizer_step
        if not self.save_dir:  # ckpt_dir=None disables checkpoint files
            return
        with context.executor.checkpoint_context(context.model) as sd:
            if sd is not None:
                path = os.path.join(self.save_dir, f"epoch_{context.epoch}_step_{context.optimizer_step}")
                extra = {} if self.weight_only else self.save_extra_fn(context)
                context.checkpoint = Checkpoint(state_dict=sd, epoch=context.epoch,
                                                consumed_samples=context.consumed_samples,
                                                config=context.model_config, extra=extra,
                                                meta=context.config.to_dict())
                context.checkpoint.save(path)
        opt = getattr(context, "optimizer", None)
        if not self.weight_only and opt is not None and getattr(opt, "sharded", False):
            # every rank holds a different optimizer shard: one file per rank next to optimizer.pt
            path = os.path.join(self.save_dir, f"epoch_{context.epoch}_step_{context.optimizer_step}")
            os.makedirs(path, exist_ok=True)
            torch.save(opt.state_dict(), os.path.join(path, f"optimizer.rank{context.rank}.pt"))
            if dist.is_available() and dist.is_initialized():
                dist.barrier()

    def on_batch_end(self, context):
        if context.optimizer_step - self.last_ckpt_step >= self.interval:
            self._save(context)

    def on_train_end(self, context):
        if context.optimizer_step != self.last_ckpt_step:
            self._save(context)

    def on_error(self, context):
        self._save(context)

    @staticmethod
    def save_extra(context) -> dict:
        out = {}
        for name in CheckpointCallback.extra_keys:
            obj = getattr(context, name, None)
            if obj:
                out[name] = obj.state_dict()
        return out


@CallbackFactory.register("progress_bar")
class ProgressBarCallback:
    def __init__(self, num_epoch: int, log_interval: int = 100, file: Optional[IO[str]] = None):
        self.num_epoch = num_epoch
        self.log_interval = log_interval
        self.file = file
        self.bar = None

    @only_on_rank(0)
    def on_epoch_begin(self, context):
        from tqdm import tqdm

        total = len(context.dataloader) // context.executor.grad_accum_steps
        self.bar = tqdm(total=total, desc=f"Epoch {context.epoch + 1}/{self.num_epoch}", dynamic_ncols=True,
                        file=self.file or sys.stdout, mininterval=2.0)

    @only_on_rank(0)
    def on_optimizer_step(self, context):
        if self.bar is None:
            return
        post = {"step": f"{context.optimizer_step:d}", "loss": f"{context.loss:.4f}",
                "lr": f"{context.optimizer.param_groups[-1]['lr']:.2e}"}
        if context.grad_norm is not None:
            post["grad_norm"] = f"{context.grad_norm:.2f}"
        if context.val_loss is not None:
            post["val_loss"] = f"{context.val_loss:.4f}"
        self.bar.set_postfix(post, refresh=False)
        self.bar.update(1)

    @only_on_rank(0)
    def on_epoch_end(self, context):
        if self.bar:
            self.bar.close()


@CallbackFactory.register("metric")
class MetricCallback:
    def __init__(self, log_dir: str, save_interval: int, metrics: Optional[List[str]] = None, val_step: int = 0):
        self.last_flush = None
        self.save_interval = save_interval
        self.metrics = metrics or ["loss", "lr"]
        self.val_step = val_step
        self._next_val = 0
        self.log_dir = Path(log_dir) if log_dir else Path.cwd() / "logs"
        self.log_dir.mkdir(parents=True, exist_ok=True)
        self.cache: List[dict] = []
        self._funcs = {
            "loss": lambda c: c.loss,
            "lr": lambda c: c.optimizer.param_groups[-1]["lr"] if c.optimizer is not None else None,
            "grad_norm": lambda c: c.grad_norm,
            "val_loss": lambda c: c.val_loss,
            "tokens_per_s": lambda c: self._rate(c)[0],
            "mfu": lambda c: self._rate(c)[1],
        }
        self._t_last = None
        self._tok_last = 0
        self._rate_cache = (None, None, -1)

    # B200 dense bf16 tensor peak per GPU (nominal), the denominator of the logged MFU
    PEAK_FLOPS = 2.25e15

    def _rate(self, c):
        """(whole-job tokens/s since the previous optimizer step, model FLOPs utilisation per GPU)."""
        if self._rate_cache[2] == c.optimizer_step:
            return self._rate_cache[:2]
        now, tok = time.perf_counter(), c.kwargs.get("tokens", 0)
        tps = mfu = None
        if self._t_last is not None and now > self._t_last and tok > self._tok_last:
            tps = (tok - self._tok_last) / (now - self._t_last)
            model = getattr(c.model, "module", c.model)
            n_params = sum(p.numel() for p in model.parameters())
            mfu = 6.0 * n_params * tps / max(1, c.world_size) / self.PEAK_FLOPS
        self._t_last, self._tok_last = now, tok
        self._rate_cache = (tps, mfu, c.optimizer_step)
        return tps, mfu

    def _append(self, kind, context, **extra):
        if context.rank != 0:
            return
        self.cache.append({"type": kind, "timestamp": time.strftime("%Y-%m-%dT%H:%M:%S"), "epoch": context.epoch,
                           "step": context.optimizer_step, "consumed_samples": context.consumed_samples, **extra})

    def _validate(self, context) -> float:
        context.model.eval()
        total = torch.zeros((), device=get_current_device(), dtype=torch.float64)
        n = 0
        with torch.no_grad():
            for batch in context.val_dataloader:
                total += context.strategy(batch).double()
                n += 1
        stats = torch.stack([total, torch.tensor(float(n), device=total.device, dtype=torch.float64)])
        if context.world_size > 1 and dist.is_initialized():
            dist.all_reduce(stats, op=dist.ReduceOp.SUM)
        context.model.train()
        return float(stats[0] / stats[1].clamp(min=1.0))

    def on_train_begin(self, context):
        self.last_flush = context.optimizer_step
        self._t_last, self._tok_last = time.perf_counter(), context.kwargs.get("tokens", 0)

    @only_on_rank(0)
    def _flush(self, epoch, step):
        f = self.log_dir / f"epoch_{epoch}_step_{step}_metric.jsonl"
        with open(f, "w") as fh:
            for e in self.cache:
                fh.write(json.dumps(e) + "\n")

    def on_optimizer_step(self, context):
        if context.val_dataloader is not None and self.val_step > 0 and context.optimizer_step >= self._next_val:
            context.val_loss = self._validate(context)
            self._next_val = context.optimizer_step + self.val_step
            self._append("validation", context, val_loss=context.val_loss)
        vals = {}
        for m in self.metrics:
            if m == "val_loss" or m not in self._funcs:
                continue
            v = self._funcs[m](context)
            if v is not None:
                vals[m] = v
        self._append("step", context, **vals)
        if context.optimizer_step - self.last_flush >= self.save_interval:
            self._flush(context.epoch, context.optimizer_step)
            self.last_flush = context.optimizer_step

    def on_epoch_end(self, context):
        self._append("epoch", context)

    def on_train_end(self, context):
        if self.last_flush is None or context.optimizer_step != self.last_flush:
            self._flush(context.epoch, context.optimizer_step)
            self.last_flush = context.optimizer_step

    def on_error(self, context):
        self._flush(context.epoch, context.optimizer_step)


@CallbackFactory.register("gradient_clipping")
class GradientClippingCallback:
    def __init__(self, max_grad_norm: Optional[float]):
        self.max_grad_norm = max_grad_norm

    def on_optimizer_step(self, context):
        # always computed: the norm is logged; clipping only if a max is set
        context.grad_norm_tensor = context.executor.clip_grad_norm(context.model, self.max_grad_norm, as_tensor=True)


@contextmanager
def nvtx_range(name: str):
    """NVTX range on CUDA (visible in Nsight / torch.profiler traces); no-op on CPU."""
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


@CallbackFactory.register("profiler")
class ProfilerCallback:
    """torch.profiler over a window of optimizer steps (skip ``wait``, warm ``warmup``,
    record ``active``); rank 0 writes a Chrome trace + a kernel table to ``profile_dir``."""

    def __init__(self, profile_dir: str, wait: int = 2, warmup: int = 1, active: int = 2):
        self.profile_dir, self.wait, self.warmup, self.active = profile_dir, wait, warmup, active
        self._prof = None

    def on_train_begin(self, context) -> None:
        from torch.profiler import ProfilerActivity, profile, schedule

        if get_rank() != 0:
            return
        os.makedirs(self.profile_dir, exist_ok=True)
        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])

        def done(p):
            p.export_chrome_trace(os.path.join(self.profile_dir, f"trace_step{p.step_num}.json"))
            sort = "cuda_time_total" if torch.cuda.is_available() else "cpu_time_total"
            with open(os.path.join(self.profile_dir, "kernels.txt"), "w") as fh:
                fh.write(p.key_averages().table(sort_by=sort, row_limit=40))

        self._prof = profile(activities=acts, schedule=schedule(wait=self.wait, warmup=self.warmup,
                                                                active=self.active, repeat=1), on_trace_ready=done)
        self._prof.__enter__()

    def on_optimizer_step(self, context) -> None:
        if self._prof is not None:
            self._prof.step()

    def on_train_end(self, context) -> None:
        if self._prof is not None:
            self._prof.__exit__(None, None, None)
            self._prof = None


@CallbackFactory.register("health")
class HealthCallback:
    """Peer failure detection for multi-rank training (no-op on one rank).

    Starts a store heartbeat when training begins, checks the peers before each
    batch (at most once per ``check_every`` seconds, a few store reads), records
    this rank's failure from ``on_error`` so the other ranks raise
    :class:`astrai_b200.parallel.health.PeerFailure` with the cause before their
    next collective instead of waiting for the process-group timeout."""

    def __init__(self, interval: float = 1.0, timeout: float = 30.0, check_every: float = 2.0):
        self.interval, self.timeout, self.check_every = interval, timeout, check_every
        self.hb = None
        self._last = 0.0

    def on_train_begin(self, context) -> None:
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            from astrai_b200.parallel.health import Heartbeat

            self.hb = Heartbeat(interval=self.interval, timeout=self.timeout).start()

    def on_batch_begin(self, context) -> None:
        if self.hb is not None and time.monotonic() - self._last >= self.check_every:
            self._last = time.monotonic()
            self.hb.check()

    def on_error(self, context) -> None:
        if self.hb is not None:
            err = sys.exc_info()[1]
            self.hb.mark_failed(repr(err) if err is not None else "error")

    def on_train_end(self, context) -> None:
        if self.hb is not None:
            self.hb.stop()
            self.hb = None
