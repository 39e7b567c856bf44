"""Training context and its builder (parity: astrai/trainer/train_context.py:22-269).

The builder creates the executor, loads a checkpoint (``param_path``; with
``resume`` also epoch / consumed samples rounded down to an optimizer-step
multiple, and optimizer / scheduler state), injects LoRA before wrapping,
builds the resumable ``RDSampler`` + DataLoader (optional validation split),
creates frozen reference / old-policy models for dpo / grpo, the strategy,
and for ``online_*`` strategies the rollout generator + runner on top of the
inference scheduler.

``TrainContext.loss`` / ``grad_norm`` are read lazily from device tensors so
the hot loop never synchronises with the host per micro-batch.
"""

from __future__ import annotations

import os

from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Dict, Optional

import torch
import torch.nn as nn
from torch.utils.data import DataLoader, random_split

from astrai_b200.config.train_config import TrainConfig
from astrai_b200.dataset.sampler import RDSampler
from astrai_b200.models.components.lora import inject_lora
from astrai_b200.parallel.executor import BaseExecutor, ExecutorFactory
from astrai_b200.parallel.setup import get_current_device, get_rank, get_world_size
from astrai_b200.serialization import Checkpoint, load_json
from astrai_b200.trainer.strategy import BaseStrategy, StrategyFactory, create_ref_model


@dataclass
class TrainContext:
    model: nn.Module = None
    strategy: BaseStrategy = None
    dataloader: DataLoader = None
    optimizer: Any = None
    scheduler: Any = None
    checkpoint: Checkpoint = None
    config: TrainConfig = None
    model_config: dict = field(default_factory=dict)
    executor: BaseExecutor = None
    epoch: int = 0
    consumed_samples: int = 0
    loss_tensor: Optional[torch.Tensor] = None
    grad_norm_tensor: Optional[torch.Tensor] = None
    val_dataloader: Optional[DataLoader] = None
    val_loss: Optional[float] = None
    world_size: int = 1
    rank: int = 0
    kwargs: Dict[str, Any] = field(default_factory=dict)

    @property
    def loss(self) -> float:
        t = self.loss_tensor
        return float(t.detach()) if isinstance(t, torch.Tensor) else (t if t is not None else 0.0)

    @loss.setter
    def loss(self, v) -> None:
        self.loss_tensor = v

    @property
    def grad_norm(self) -> Optional[float]:
        t = self.grad_norm_tensor
        return float(t) if isinstance(t, torch.Tensor) else t

    @grad_norm.setter
    def grad_norm(self, v) -> None:
        self.grad_norm_tensor = v

    @property
    def optimizer_step(self) -> int:
        return self.consumed_samples // (self.config.batch_per_device * self.world_size * self.config.grad_accum_steps)


class TrainContextBuilder:
    def __init__(self, config: TrainConfig):
        self.config = config
        self._param_path: Optional[str] = None
        self._resume = False

    def with_param_path(self, param_path: Optional[str], resume: bool = False) -> "TrainContextBuilder":
        self._param_path = param_path
        self._resume = resume
        return self

    def build(self) -> TrainContext:
        cfg = self.config
        device = get_current_device()
        world = get_world_size()
        ekw = dict(cfg.executor_kwargs)
        if cfg.parallel_mode == "ddp":
            ekw.setdefault("comm_backend", "fused" if cfg.comm_backend == "fused" else "nccl")
        executor = ExecutorFactory.create(cfg.parallel_mode, grad_accum_steps=cfg.grad_accum_steps, **ekw)

        model_config: dict = {}
        if self._param_path and (Path(self._param_path) / "config.json").exists():
            model_config = load_json(Path(self._param_path) / "config.json")
        sd = None
        epoch = cfg.start_epoch
        consumed = cfg.start_samples * world
        ckpt = None
        if self._param_path:
            c = Checkpoint.load_any(self._param_path)
            if c is not None:
                sd = c.state_dict
                if c.config:
                    model_config = c.config
                if self._resume:
                    epoch = c.epoch or cfg.start_epoch
                    per_step = cfg.batch_per_device * world * cfg.grad_accum_steps
                    consumed = (c.consumed_samples // per_step) * per_step if c.consumed_samples > 0 \
                        else cfg.start_samples * world
                    ckpt = c
        if not model_config:
            m = cfg.model_fn()
            if hasattr(m, "config") and hasattr(m.config, "to_dict"):
                model_config = m.config.to_dict()
            del m

        def before_wrap(m):
            m = m.to(device=device)
            if cfg.lora is not None:
                inject_lora(m, r=cfg.lora.r, alpha=cfg.lora.alpha, target_modules=set(cfg.lora.target_modules))
            if sd is not None:
                m.load_state_dict(sd, strict=False)
            return m

        ctx = TrainContext(world_size=world, rank=get_rank(), config=cfg, model_config=model_config,
                           executor=executor, epoch=epoch, consumed_samples=consumed, checkpoint=ckpt)
        ctx.model, ctx.optimizer, ctx.scheduler = executor.prepare(cfg.model_fn, cfg.optimizer_fn, cfg.scheduler_fn,
                                                                    before_wrap=before_wrap)
        if cfg.neftune_alpha and hasattr(executor.unwrap(ctx.model), "embed_tokens"):
            executor.unwrap(ctx.model).embed_tokens.set_neftune_alpha(cfg.neftune_alpha)

        train_ds, val_ds = cfg.dataset, cfg.val_dataset
        if val_ds is None and cfg.val_split is not None:
            n = len(cfg.dataset)
            nv = max(1, int(n * cfg.val_split))
            train_ds, val_ds = random_split(cfg.dataset, [n - nv, nv],
                                            generator=torch.Generator().manual_seed(cfg.random_seed))
        sampler = RDSampler(train_ds, start_epoch=ctx.epoch, start_iter=ctx.consumed_samples // ctx.world_size,
                            seed=cfg.random_seed)
        dl_kw = dict(num_workers=cfg.num_workers, pin_memory=cfg.pin_memory, collate_fn=cfg.collate_fn)
        if cfg.num_workers > 0 and cfg.prefetch_factor is not None:
            dl_kw["prefetch_factor"] = cfg.prefetch_factor
        ctx.dataloader = DataLoader(train_ds, batch_size=cfg.batch_per_device, sampler=sampler, **dl_kw)
        if val_ds is not None:
            vs = RDSampler(val_ds, start_epoch=0, start_iter=0, seed=cfg.random_seed, shuffle=False)
            ctx.val_dataloader = DataLoader(val_ds, batch_size=cfg.batch_per_device, sampler=vs, **dl_kw)

        if ctx.checkpoint is not None and ctx.checkpoint.extra:
            for name in ("optimizer", "scheduler"):
                obj = getattr(ctx, name, None)
                if obj is not None and name in ctx.checkpoint.extra:
                    obj.load_state_dict(ctx.checkpoint.extra[name])
        shard_file = os.path.join(str(self._param_path), f"optimizer.rank{ctx.rank}.pt") \
            if self._param_path and self._resume else None
        if ctx.optimizer is not None and getattr(ctx.optimizer, "sharded", False) and shard_file \
                and os.path.exists(shard_file):
            ctx.optimizer.load_state_dict(torch.load(shard_file, map_location="cpu", weights_only=False))

        skw = dict(cfg.extra_kwargs)
        if cfg.strategy in ("dpo", "grpo", "online_grpo", "online_dpo"):
            skw["ref_model"] = create_ref_model(cfg.model_fn, executor.unwrap_model(ctx.model)).to(device=device)
        if cfg.strategy in ("grpo", "online_grpo"):
            skw["old_model"] = create_ref_model(cfg.model_fn, executor.unwrap_model(ctx.model)).to(device=device)
        ctx.strategy = StrategyFactory.create(cfg.strategy, model=ctx.model, device=device, executor=executor, **skw)

        if cfg.strategy.startswith("online_"):
            if not ctx.strategy.supports_online():
                raise ValueError(f"Strategy '{cfg.strategy}' does not support online rollout")
            if cfg.reward_model_fn is None:
                raise ValueError("reward_model_fn is required for online RL strategies")
            from astrai_b200.inference.core.scheduler import InferenceScheduler
            from astrai_b200.tokenize import AutoTokenizer
            from astrai_b200.trainer.rollout import RolloutGenerator, RolloutRunner

            tok = AutoTokenizer.from_pretrained(self._param_path)
            group = skw.get("group_size", 1)
            base = executor.unwrap(ctx.model)
            max_len = getattr(base.config, "max_position_embeddings", None)
            sched = InferenceScheduler(model=base, tokenizer=tok, max_batch_size=group * max(1, cfg.batch_per_device),
                                       max_seq_len=max_len, max_prompt_len=max_len or 4096)
            gen = RolloutGenerator(scheduler=sched, tokenizer=tok, max_tokens=cfg.rollout_max_tokens, group_size=group,
                                   temperature=cfg.rollout_temperature, top_k=cfg.rollout_top_k,
                                   top_p=cfg.rollout_top_p)
            ctx.strategy.set_rollout_runner(RolloutRunner(generator=gen, reward_model=cfg.reward_model_fn(),
                                                          rollout_interval=cfg.rollout_interval))
        return ctx
