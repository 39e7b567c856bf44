"""Metric helpers (parity: astrai/trainer/metric_util.py)."""

from typing import Iterable, Optional

import torch


def grad_norm(params: Iterable[torch.Tensor], norm_type: float = 2.0) -> float:
    gs = [p.grad.detach().float() for p in params if p.grad is not None]
    if not gs:
        return 0.0
    return float(torch.linalg.vector_norm(torch.stack([torch.linalg.vector_norm(g, norm_type) for g in gs]), norm_type))


def ctx_get_loss(ctx) -> float:
    return ctx.loss


def ctx_get_lr(ctx) -> Optional[float]:
    return ctx.optimizer.param_groups[-1]["lr"] if ctx.optimizer is not None else None


def ctx_get_grad_norm(ctx) -> Optional[float]:
    return ctx.grad_norm


def ctx_get_val_loss(ctx) -> Optional[float]:
    return ctx.val_loss
