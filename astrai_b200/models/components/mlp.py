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
The MoE runs the fused router kernel and the routed-expert block of
:mod:`astrai_b200.ops.moe` (dispatch -> batched expert GEMMs -> return ->
weighted combine fused with the residual and shared-expert sum); with
:meth:`DeepSeekMoE.shard_experts` the routed experts are split over an
expert-parallel group and token rows move over NVLink peer memory. Routed
experts live in a ModuleDict keyed by their global index, so state-dict keys
stay ``routed_experts.{j}...`` (a sharded layer holds its own experts only).
"""

from __future__ import annotations

import os

from typing import Optional

import torch
import torch.nn as nn

from astrai_b200.factory import Registry
from astrai_b200.models.components.basic import Linear
from astrai_b200.ops.activation import swiglu
from astrai_b200.ops.gemm import linear, packed_linear, swiglu_mlp


class FFNFactory(Registry[nn.Module]):
    pass


@FFNFactory.register("mlp")
class MLP(nn.Module):
    def __init__(self, dim: int, dim_ffn: int, down_init_std: float = 0.02):
        super().__init__()
        self.up = Linear(dim, dim_ffn)
        self.gate = Linear(dim, dim_ffn)
        self.down = Linear(dim_ffn, dim, init_std=down_init_std)

    def packed_groups(self):
        """Parameters the kernel path packs into one buffer (up then gate: one GEMM)."""
        if type(self.up) is Linear and type(self.gate) is Linear and self.up.bias is None and self.gate.bias is None:
            return [[self.up.weight, self.gate.weight]]
        return []

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None, ctx=None) -> torch.Tensor:
        plain = all(type(m) is Linear and m.bias is None for m in (self.up, self.gate, self.down))
        if plain:
            y = swiglu_mlp(x, self.up.weight, self.gate.weight, self.down.weight, residual)
            if y is not None:
                return y
        if type(self.up) is Linear and type(self.gate) is Linear and self.up.bias is None and self.gate.bias is None:
            h = packed_linear(x, [self.up.weight, self.gate.weight])
        else:
            h = torch.cat([self.up(x), self.gate(x)], dim=-1)
        return self.down(swiglu(h), residual=residual)


@FFNFactory.register("moe")
class DeepSeekMoE(nn.Module):
    # the expert layout is built on the device (no host round trip): the micro-step can be captured in a
    # CUDA graph once the arena exists (it is sized for the token count of the first call)
    cuda_graph_safe = True
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
        self.routed_experts = nn.ModuleDict({str(j): MLP(dim, ffn, down_std) for j in range(n_routed_experts)})
        # EP arena rows per rank relative to the mean expert load; a heavier load is reported on the device
        # error word (kErrBadArg) and its rows dropped: raise it for strongly imbalanced routing
        self.capacity_factor = float(os.environ.get("ASTRAI_MOE_CAPACITY", "2.0"))
        # expert-parallel dispatch payload as fp8 e4m3 with 1x128 block scales (opt-in, halves the
        # dispatch bytes over NVLink; the reference moves no tokens between ranks at all)
        self.fp8_dispatch = os.environ.get("ASTRAI_EP_FP8", "0") == "1"
        self._ep = None
        self._arena = None
        self._stack = None

    # ------------------------------------------------------------------ expert parallelism
    def shard_experts(self, group=None) -> None:
        """Keep only this rank's experts (E / world consecutive ones) of ``group``."""
        from astrai_b200.parallel.ep import EPGroup

        ep = EPGroup(group)
        if self.n_routed_experts % ep.world:
            raise ValueError(f"{self.n_routed_experts} experts do not split over {ep.world} ranks")
        el = self.n_routed_experts // ep.world
        keep = {str(j) for j in range(ep.rank * el, (ep.rank + 1) * el)}
        self.routed_experts = nn.ModuleDict({k: m for k, m in self.routed_experts.items() if k in keep})
        for p in self.routed_experts.parameters():
            p._ep_local = True  # gradients come from every rank's tokens: no data-parallel all-reduce
        if self._arena is not None:  # sharded again (a second executor over the same model)
            self._arena.close()
        self._ep, self._arena, self._stack = ep, None, None

    @property
    def expert_parallel(self) -> bool:
        return self._ep is not None and self._ep.world > 1

    def packed_groups(self):
        """The routed experts' stacked weights (all up / gate rows, all down rows) and the shared
        experts' up / gate pairs."""
        groups = [g for e in self.shared_experts for g in e.packed_groups()]
        experts = list(self.routed_experts.values())
        if experts and all(type(m.up) is Linear and type(m.gate) is Linear and type(m.down) is Linear
                           for m in experts):
            groups.append([w for m in experts for w in (m.up.weight, m.gate.weight)])
            groups.append([m.down.weight for m in experts])
        return groups

    def _fused_ok(self, x: torch.Tensor) -> bool:
        from astrai_b200.ops import gemm as _gemm

        experts = list(self.routed_experts.values())
        return (_gemm.PACKING and x.is_cuda and x.dtype == torch.bfloat16 and self.dim % 8 == 0 and self.n_activated_experts <= 8
                and self.n_routed_experts <= 256 and all(type(m.up) is Linear and type(m.down) is Linear
                                                         and m.up.weight.dtype == torch.bfloat16 for m in experts))

    def route(self, x: torch.Tensor):
        """Router: fp32 softmax -> top-k -> renormalised weights (+ balance stats)."""
        logits = linear(x, self.router.weight) if x.is_cuda else self.router(x)
        probs = torch.softmax(logits.float(), dim=-1)
        w, idx = torch.topk(probs.to(x.dtype), self.n_activated_experts, dim=-1)
        w = w / w.sum(dim=-1, keepdim=True)
        return probs, w, idx

    def _shared(self, xf: torch.Tensor) -> Optional[torch.Tensor]:
        if not self.n_shared_experts:
            return None
        sh = sum(e(xf) for e in self.shared_experts)
        return sh / self.n_shared_experts if self.shared_mode == "mean" else sh

    def _forward_fused(self, xf: torch.Tensor, residual: Optional[torch.Tensor], ctx) -> torch.Tensor:
        from astrai_b200.ops.moe import moe_experts, moe_route, stack_expert_params
        from astrai_b200.parallel.ep import EPArena, EPGroup, EPLayout

        T, d = xf.shape
        k = self.n_activated_experts
        logits = linear(xf, self.router.weight)
        w, probs, idx, counts, pos = moe_route(logits, k)
        if self._ep is None:  # not sharded: this rank runs all experts on its own tokens
            self._ep = EPGroup.local()
        ep = self._ep
        if self._arena is None or self._arena.slots_cap < T * k:
            if self._arena is not None:
                self._arena.close()
            self._arena = EPArena(ep, d, T, k, self.n_routed_experts, self.capacity_factor, xf.device,
                                  fp8=self.fp8_dispatch)
        # counts exchange + layout on the device: nothing is read back, so the layer can be graphed
        layout = self._arena.compute_layout(counts)
        self._stack = stack_expert_params(self.routed_experts.values())
        add = self._shared(xf)
        if residual is not None:
            r = residual.reshape(-1, d)
            add = r if add is None else add + r
        if add is not None:
            add = add.contiguous()
        out = moe_experts(xf.contiguous(), add, w, idx, pos, self._stack, self._arena, layout)
        if self.aux_loss_coef > 0 and self.training and ctx is not None and ctx.aux_losses is not None:
            f = counts.float() / max(1, T * k)
            ctx.aux_losses.append(self.aux_loss_coef * self.n_routed_experts * (f * probs.mean(0)).sum())
        return out

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None, ctx=None) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, shape[-1])
        if self._fused_ok(xf):
            return self._forward_fused(xf, residual, ctx).view(shape)
        if self.expert_parallel:
            raise RuntimeError("expert-parallel MoE needs CUDA bf16 activations")
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
            y = self.routed_experts[str(e)](xf[t]) * wts[start:start + c]
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
