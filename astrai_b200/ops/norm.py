"""RMSNorm (parity: astrai/model/components/norm.py:7-15, ``F.rms_norm``)."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from astrai_b200.ops._ext import native


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.stride(-1) != 1 or (x2.stride(0) * 2) % 16:
            x2 = x2.contiguous()
        y = torch.empty((x2.shape[0], shape[-1]), device=x.device, dtype=x.dtype)
        rstd = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        native().rmsnorm_fwd(x2, w, y, rstd, float(eps))
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        C = native()
        dy2 = dy.reshape(-1, x2.shape[1])
        if dy2.stride(-1) != 1 or (dy2.stride(0) * 2) % 16:
            dy2 = dy2.contiguous()
        dx = torch.empty_like(x2)
        dw = torch.empty_like(w)
        scratch = torch.empty(C.rmsnorm_bwd_scratch(x2.shape[0], x2.shape[1]), device=x2.device, dtype=torch.float32)
        C.rmsnorm_bwd(dy2, x2, w, rstd, dx, dw, scratch)
        return dx.view(ctx.shape), dw, None


class _RMSNormForkFn(torch.autograd.Function):
    """``(rms_norm(x), x)`` for a pre-norm block that also feeds x to its residual add: the gradient
    arriving through the second output is added to dx inside the norm backward kernel, instead of
    autograd summing the two branches with a separate elementwise kernel."""

    @staticmethod
    def forward(ctx, x, w, eps):
        y = _RMSNormFn.forward(ctx, x, w, eps)
        return y, x

    @staticmethod
    def backward(ctx, dy, dres):
        x2, w, rstd = ctx.saved_tensors
        C = native()
        D = x2.shape[1]
        if dy is None:
            return dres, None, None
        dy2 = dy.reshape(-1, D)
        if dy2.stride(-1) != 1 or (dy2.stride(0) * 2) % 16:
            dy2 = dy2.contiguous()
        r2 = None
        if dres is not None:
            r2 = dres.reshape(-1, D)
            if r2.stride(-1) != 1 or (r2.stride(0) * 2) % 16:
                r2 = r2.contiguous()
        dx = torch.empty_like(x2)
        dw = torch.empty_like(w)
        scratch = torch.empty(C.rmsnorm_bwd_scratch(x2.shape[0], D), device=x2.device, dtype=torch.float32)
        C.rmsnorm_bwd(dy2, x2, w, rstd, dx, dw, scratch, r2)
        return dx.view(ctx.shape), dw, None


def _fast(x: torch.Tensor, weight: torch.Tensor, backward: bool = True) -> bool:
    D = x.shape[-1]
    # each thread of a row's block owns fixed 8-column groups: up to 2 per thread in the backward
    # kernel (D <= 4096), 4 in the forward one (D <= 8192)
    return x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and D % 8 == 0 \
        and (D > 256 or D % 32 == 0) and D <= (4096 if backward else 8192)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    backward = torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad)
    if _fast(x, weight, backward):
        return _RMSNormFn.apply(x, weight, eps)
    return F.rms_norm(x, (x.shape[-1],), weight, eps)


def rms_norm_fork(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """``(rms_norm(x), x)``; on the kernel path the two gradients of x are summed in the norm backward."""
    if _fast(x, weight) and torch.is_grad_enabled() and x.requires_grad:
        return _RMSNormForkFn.apply(x, weight, eps)
    return rms_norm(x, weight, eps), x
