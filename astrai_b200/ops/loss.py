"""Fused cross-entropy and token log-probabilities from bf16 logits.

Parity:
* ``cross_entropy`` == ``F.cross_entropy(logits.float(), target,
  ignore_index=..., label_smoothing=...)`` with mean reduction over
  non-ignored tokens (astrai/trainer/strategy.py:215-226, :246-269);
* ``token_logprobs`` == ``log_softmax(logits.float()).gather(target)``
  (strategy.py:59-67), used by DPO / GRPO.

On CUDA no fp32 copy of the [tokens, vocab] logits is created: the kernels
stream bf16 rows and keep only the per-row log-sum-exp.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from astrai_b200.ops._ext import native


def _rows(t):
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1 or (t2.stride(0) * 2) % 16:
        t2 = t2.contiguous()
    return t2


class _CEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, smoothing, ignore_index):
        x = _rows(logits)
        t = target.reshape(-1).contiguous().long()
        lse = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        per_row = torch.empty_like(lse)
        native().ce_fwd(x, t, float(smoothing), int(ignore_index), 0, lse, per_row)
        count = (t != ignore_index).sum().clamp_min(1).float()
        loss = per_row.sum() / count
        ctx.save_for_backward(x, t, lse, count)
        ctx.smoothing, ctx.ignore = smoothing, ignore_index
        ctx.shape = logits.shape
        return loss

    @staticmethod
    def backward(ctx, g):
        x, t, lse, count = ctx.saved_tensors
        gscale = (g.float() / count).reshape(1).contiguous()
        dx = torch.empty_like(x)
        native().ce_bwd(x, t, float(ctx.smoothing), int(ctx.ignore), 0, lse, gscale, None, dx)
        return dx.view(ctx.shape), None, None, None


class _LogprobFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target):
        x = _rows(logits)
        t = target.reshape(-1).contiguous().long()
        lse = torch.empty(x.shape[0], device=x.device, dtype=torch.float32)
        lp = torch.empty_like(lse)
        native().ce_fwd(x, t, 0.0, -100, 1, lse, lp)
        ctx.save_for_backward(x, t, lse)
        ctx.shape = logits.shape
        return lp.view(target.shape)

    @staticmethod
    def backward(ctx, g):
        x, t, lse = ctx.saved_tensors
        dx = torch.empty_like(x)
        native().ce_bwd(x, t, 0.0, -100, 1, lse, None, g.reshape(-1).float().contiguous(), dx)
        return dx.view(ctx.shape), None


def _fused_ok(logits):
    return logits.is_cuda and logits.dtype == torch.bfloat16


def cross_entropy(logits: torch.Tensor, target: torch.Tensor, label_smoothing: float = 0.0,
                  ignore_index: int = -100) -> torch.Tensor:
    if _fused_ok(logits):
        return _CEFn.apply(logits, target, label_smoothing, ignore_index)
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), target.reshape(-1),
                           ignore_index=ignore_index, label_smoothing=label_smoothing)


def token_logprobs(logits: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    """log p(target) per position; logits [..., V], target [...]."""
    if _fused_ok(logits):
        return _LogprobFn.apply(logits, target)
    lp = torch.log_softmax(logits.float(), dim=-1)
    return torch.gather(lp, -1, target.unsqueeze(-1)).squeeze(-1)
