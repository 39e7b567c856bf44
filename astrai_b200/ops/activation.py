"""SwiGLU on the fused [up | gate] projection output.

Parity: astrai/model/components/mlp.py:22-25 computes ``up(x) * silu(gate(x))``
with two GEMMs; here one GEMM produces ``h = [up | gate]`` (weights
concatenated along the output dimension) and one kernel applies the gate.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from astrai_b200.ops._ext import native


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h):
        F_ = h.shape[-1] // 2
        h2 = h.reshape(-1, 2 * F_)
        out = torch.empty((h2.shape[0], F_), device=h.device, dtype=h.dtype)
        native().swiglu_fwd(h2, out)
        ctx.save_for_backward(h2)
        ctx.shape = h.shape
        return out.view(*h.shape[:-1], F_)

    @staticmethod
    def backward(ctx, dy):
        (h2,) = ctx.saved_tensors
        dy2 = dy.reshape(-1, h2.shape[1] // 2)
        if dy2.stride(-1) != 1:
            dy2 = dy2.contiguous()
        dh = torch.empty_like(h2)
        native().swiglu_bwd(dy2, h2, dh)
        return dh.view(ctx.shape)


def swiglu(h: torch.Tensor) -> torch.Tensor:
    """h = [up | gate] along the last dim -> up * silu(gate)."""
    F_ = h.shape[-1] // 2
    if h.is_cuda and h.dtype == torch.bfloat16 and F_ % 8 == 0 and h.stride(-1) == 1:
        return _SwiGLUFn.apply(h)
    up, gate = h[..., :F_], h[..., F_:]
    return up * F.silu(gate)
