"""Feed-forward modules: SwiGLU MLP and DeepSeek-style MoE.

Names follow the reference (astrai/model/components/mlp.py): MLP has ``up``,
``gate``, ``down``; the MoE has ``router``, ``shared_experts.{j}``,
``routed_experts.{j}``. Semantics kept: fp32 softmax router, top-k, weights
renormalised to sum 1, shared experts averaged, MoE down-projection init
``0.02 / sqrt(2 L (1/max(ns,1) + 1/k))``.

Additions: a switch-style balance loss ``coef * E * sum_e f_e * P_e``
(f_e = fraction of routed slots that chose expert e, P_e = mean router
probability), collected into ``AttnContext.aux_losses`` when
``aux_loss_coef > 0``; ``shared_expert_mode="sum"`` sums shared experts.

On the GPU the MLP runs up|gate as one GEMM (weights concatenated), the
SwiGLU kernel, and the down GEMM with the residual added in its epilogue.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from astrai_b200.factory import Registry
from astrai_b200.models.components.basic import Linear
from astrai_b200.ops.activation import swiglu
from astrai_b200.ops.gemm import linear, packed_linear


class FFNFactory(Registry[nn.Module]):
    pass


@FFNFactory.register("mlp")
class MLP(nn.Module):
    def __init__(self, dim: int, dim_ffn: int, down_init_std: float = 0.02):
        super().__init__()
        self.up = Linear(dim, dim_ffn)
        self.gate = Linear(dim, dim_ffn)
        self.down = Linear(dim_ffn, dim, init_std=down_init_std)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None, ctx=None) -> torch.Tensor:
        if type(self.up) is Linear and type(self.gate) is Linear and self.up.bias is None and self.gate.bias is None:
            h = packed_linear(x, [self.up.weight, self.gate.weight])
        else:
            h = torch.cat([self.up(x), self.gate(x)], dim=-1)
        return self.down(swiglu(h), residual=residual)


@FFNFactory.register("moe")
class DeepSeekMoE(nn.Module):
    def __init__(self, dim: int, dim_ffn: int, n_routed_experts: int, n_shared_experts: int = 1,
                 n_activated_experts: int = 2, topk_method: str = "greedy", n_layers: int = 1,
                 moe_intermediate_size: Optional[int] = None, moe_aux_loss_coef: Optional[float] = None,
                 shared_expert_mode: Optional[str] = None):
        super().__init__()
        self.dim = dim
        self.n_routed_experts = n_routed_experts
        self.n_shared_experts = n_shared_experts or 0
        self.n_activated_experts = n_activated_experts
        self.topk_method = topk_method
        self.aux_loss_coef = float(moe_aux_loss_coef or 0.0)
        self.shared_mode = shared_expert_mode or "mean"
        ffn = moe_intermediate_size or dim_ffn
        self.router = Linear(dim, n_routed_experts)
        moe_scale = 1.0 / max(self.n_shared_experts, 1) + 1.0 / n_activated_experts
        down_std = 0.02 / (2 * n_layers * moe_scale) ** 0.5
        self.shared_experts = nn.ModuleList([MLP(dim, ffn, down_std) for _ in range(self.n_shared_experts)])
        self.routed_experts = nn.ModuleList([MLP(dim, ffn, down_std) for _ in range(n_routed_experts)])

    def route(self, x: torch.Tensor):
        """Router: fp32 softmax -> top-k -> renormalised weights (+ balance stats)."""
        logits = linear(x, self.router.weight) if x.is_cuda else self.router(x)
        probs = torch.softmax(logits.float(), dim=-1)
        w, idx = torch.topk(probs.to(x.dtype), self.n_activated_experts, dim=-1)
        w = w / w.sum(dim=-1, keepdim=True)
        return probs, w, idx

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None, ctx=None) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        N = xf.shape[0]
        probs, w, idx = self.route(xf)
        out = torch.zeros_like(xf)
        # group tokens by expert (one sort instead of E nonzero scans)
        flat_e = idx.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        counts = torch.bincount(flat_e, minlength=self.n_routed_experts).tolist()
        tok = order // self.n_activated_experts
        wts = w.reshape(-1)[order].unsqueeze(-1)
        start = 0
        for e, c in enumerate(counts):
            if c == 0:
                continue
            t = tok[start:start + c]
            y = self.routed_experts[e](xf[t]) * wts[start:start + c]
            out = out.index_add(0, t, y.to(out.dtype))
            start += c
        if self.n_shared_experts:
            sh = sum(e(xf) for e in self.shared_experts)
            out = out + (sh / self.n_shared_experts if self.shared_mode == "mean" else sh)
        if self.aux_loss_coef > 0 and self.training and ctx is not None and ctx.aux_losses is not None:
            f = torch.bincount(flat_e, minlength=self.n_routed_experts).float() / max(1, flat_e.numel())
            P = probs.mean(0)
            ctx.aux_losses.append(self.aux_loss_coef * self.n_routed_experts * (f * P).sum())
        out = out.view(shape)
        return out + residual if residual is not None else out
