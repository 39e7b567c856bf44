"""Attention modules: GQA and MLA.

Parameter names follow the reference (astrai/model/components/attention.py:30-213):
GQA has ``q_proj, k_proj, v_proj, o_proj`` (+ ``q_norm, k_norm`` for QK-norm,
``gate`` for gated attention); MLA has ``q_proj, kv_a_proj, kv_norm,
kv_b_proj, o_proj`` (+ ``gate``). Semantics kept: RoPE on q/k, QK-norm
applied after RoPE, sigmoid output gate, o_proj init std 0.02/sqrt(2L).

Execution differs: on the GPU the three projections run as ONE GEMM over the
concatenated weight (autograd splits the weight gradient back), RoPE is
applied in place on that buffer and the flash-attention kernels read q/k/v
straight out of it; the o-projection adds the residual in its epilogue.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Optional

import torch
import torch.nn as nn

from astrai_b200.factory import Registry
from astrai_b200.models.components.basic import Linear, RMSNorm
from astrai_b200.ops.attention import attention, attention_qkv, attention_reference
from astrai_b200.ops.rope import apply_rope_reference


@dataclass
class AttnContext:
    """Per-forward attention metadata shared by all layers."""

    B: int
    S: int
    table: torch.Tensor                      # fp32 (cos, sin) [max_pos, d/2, 2]
    positions: Optional[torch.Tensor] = None  # [B, S] int, None -> arange
    seg: Optional[torch.Tensor] = None        # [B, S] int32 segment ids (docs / padding)
    dense_mask: Optional[torch.Tensor] = None  # bool [B, 1, S, Sk] (generic fallback)
    causal: bool = True
    cache: Any = None                        # inference cache view with .attend()
    aux_losses: Optional[list] = None         # MoE balance losses collected here

    def rope_rows(self) -> torch.Tensor:
        if self.positions is None:
            return self.table[: self.S].unsqueeze(0).expand(self.B, -1, -1, -1)
        return self.table[self.positions]


def _dense_attention(q, k, v, mask):
    """Arbitrary boolean mask [B,1,Sq,Sk] (reference-compatible generic path)."""
    import math

    B, Sq, Hq, D = q.shape
    Hkv = k.shape[2]
    rep = Hq // Hkv
    kk = k.repeat_interleave(rep, 2) if rep > 1 else k
    vv = v.repeat_interleave(rep, 2) if rep > 1 else v
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), kk.float()) / math.sqrt(D)
    s = s.masked_fill(~mask.bool(), float("-inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    return torch.einsum("bhqk,bkhd->bqhd", p, vv.float()).to(q.dtype)


class AttnFactory(Registry[nn.Module]):
    pass


@AttnFactory.register("gqa")
class GQA(nn.Module):
    def __init__(self, dim: int, n_heads: int, n_kv_heads: int, use_qk_norm: bool = False, norm_eps: float = 1e-6,
                 use_gated_attention: bool = False, layer_id: int = 0, n_layers: int = 1):
        super().__init__()
        assert dim % n_heads == 0 and n_heads % n_kv_heads == 0
        self.dim, self.n_heads, self.n_kv_heads = dim, n_heads, n_kv_heads
        self.head_dim = dim // n_heads
        self.layer_id = layer_id
        self.use_qk_norm = bool(use_qk_norm)
        self.use_gated_attention = bool(use_gated_attention)
        self.q_proj = Linear(dim, n_heads * self.head_dim)
        self.k_proj = Linear(dim, n_kv_heads * self.head_dim)
        self.v_proj = Linear(dim, n_kv_heads * self.head_dim)
        self.o_proj = Linear(dim, dim, init_std=0.02 / (2 * n_layers) ** 0.5)
        if self.use_qk_norm:
            self.q_norm = RMSNorm(self.head_dim, norm_eps)
            self.k_norm = RMSNorm(self.head_dim, norm_eps)
        if self.use_gated_attention:
            self.gate = Linear(dim, dim)

    def qkv_weight(self) -> torch.Tensor:
        return torch.cat([self.q_proj.weight, self.k_proj.weight, self.v_proj.weight], 0)

    def forward(self, x: torch.Tensor, ctx: AttnContext, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, _ = x.shape
        Hq, Hkv, D = self.n_heads, self.n_kv_heads, self.head_dim
        fused = not self.use_qk_norm and ctx.dense_mask is None
        if fused and ctx.cache is not None:  # inference: the cache view runs RoPE + KV write + attention
            fused = getattr(ctx.cache, "supports_qkv", False) and x.is_cuda and x.dtype == torch.bfloat16
        if fused:
            qkv = None
            if ctx.cache is None:  # training: RoPE in the QKV projection epilogue
                qkv = self.qkv_proj_rope(x, ctx)
            rotated = qkv is not None
            if qkv is None:
                qkv = self.qkv_proj(x)
            qkv = qkv.reshape(B * S, (Hq + 2 * Hkv) * D)
            if ctx.cache is not None:
                o = ctx.cache.attend_qkv(self.layer_id, qkv, B, S, Hq, Hkv, ctx.table)
            else:
                o = attention_qkv(qkv, B, S, Hq, Hkv, ctx.table, ctx.positions, ctx.causal, ctx.seg,
                                  rotated=rotated)
            o = o.view(B, S, Hq * D)
        else:
            qkv = self.qkv_proj(x)
            q, k, v = qkv.view(B, S, Hq + 2 * Hkv, D).split([Hq, Hkv, Hkv], dim=2)
            cs = ctx.rope_rows()
            q, k = apply_rope_reference(q, cs), apply_rope_reference(k, cs)
            if self.use_qk_norm:
                q, k = self.q_norm(q), self.k_norm(k)
            if ctx.cache is not None:
                o = ctx.cache.attend(self.layer_id, q, k, v.contiguous())
            elif ctx.dense_mask is not None:
                o = _dense_attention(q, k, v, ctx.dense_mask)
            else:
                o = attention(q, k, v, causal=ctx.causal, seg=ctx.seg)
            o = o.reshape(B, S, Hq * D)
        if self.use_gated_attention:
            o = o * torch.sigmoid(self.gate(x))
        return self.o_proj(o, residual=residual)

    def qkv_proj_rope(self, x: torch.Tensor, ctx) -> Optional[torch.Tensor]:
        """q|k|v projection with RoPE already applied to q and k (GEMM epilogue), or None."""
        mods = (self.q_proj, self.k_proj, self.v_proj)
        if not all(type(m) is Linear and m.bias is None for m in mods) or self.head_dim % 32:
            return None
        from astrai_b200.ops.gemm import packed_linear_rope

        pos = ctx.positions.reshape(-1).to(torch.int32).contiguous() if ctx.positions is not None else None
        return packed_linear_rope(x, [m.weight for m in mods], ctx.table, pos, ctx.S,
                                  (self.n_heads + self.n_kv_heads) * self.head_dim, self.head_dim)

    def packed_groups(self):
        """q, k and v projection weights: packed into one buffer for one GEMM."""
        mods = (self.q_proj, self.k_proj, self.v_proj)
        if all(type(m) is Linear and m.bias is None for m in mods):
            return [[m.weight for m in mods]]
        return []

    def qkv_proj(self, x: torch.Tensor) -> torch.Tensor:
        """q|k|v projections as one GEMM over the concatenated weight (plain
        Linear layers), else per-module calls (LoRA-wrapped or biased)."""
        mods = (self.q_proj, self.k_proj, self.v_proj)
        if all(type(m) is Linear and m.bias is None for m in mods):
            from astrai_b200.ops.gemm import packed_linear

            return packed_linear(x, [m.weight for m in mods])
        return torch.cat([m(x) for m in mods], dim=-1)


@AttnFactory.register("mla")
class MLA(nn.Module):
    """Multi-head latent attention: low-rank KV (kv_a_proj -> RMSNorm -> kv_b_proj),
    RoPE on the rope part of q/k only, decompressed k/v cached."""

    def __init__(self, dim: int, n_heads: int, n_kv_heads: int, kv_lora_rank: int, qk_nope_head_dim: int,
                 qk_rope_head_dim: int, norm_eps: float = 1e-6, use_qk_norm: bool = False,
                 use_gated_attention: bool = False, layer_id: int = 0, n_layers: int = 1):
        super().__init__()
        self.dim, self.n_heads, self.n_kv_heads = dim, n_heads, n_kv_heads
        self.kv_lora_rank = kv_lora_rank
        self.qk_nope_head_dim, self.qk_rope_head_dim = qk_nope_head_dim, qk_rope_head_dim
        self.head_dim = qk_nope_head_dim + qk_rope_head_dim
        self.layer_id = layer_id
        self.use_qk_norm = bool(use_qk_norm)
        self.use_gated_attention = bool(use_gated_attention)
        self.q_proj = Linear(dim, n_heads * self.head_dim)
        if self.use_qk_norm:
            self.q_norm = RMSNorm(self.head_dim, norm_eps)
            self.k_norm = RMSNorm(self.head_dim, norm_eps)
        self.kv_a_proj = Linear(dim, kv_lora_rank)
        self.kv_norm = RMSNorm(kv_lora_rank, norm_eps)
        self.kv_b_proj = Linear(kv_lora_rank, n_kv_heads * 2 * self.head_dim)
        self.o_proj = Linear(dim, dim, init_std=0.02 / (2 * n_layers) ** 0.5)
        if self.use_gated_attention:
            self.gate = Linear(dim, dim)

    def forward(self, x: torch.Tensor, ctx: AttnContext, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, _ = x.shape
        H, Hkv, D = self.n_heads, self.n_kv_heads, self.head_dim
        nope, rope = self.qk_nope_head_dim, self.qk_rope_head_dim
        q = self.q_proj(x).view(B, S, H, D)
        kv = self.kv_b_proj(self.kv_norm(self.kv_a_proj(x))).view(B, S, Hkv, 2 * D)
        k_nope, k_rope, v = torch.split(kv, [nope, rope, D], dim=-1)
        cs = ctx.rope_rows()
        q = torch.cat([q[..., :nope], apply_rope_reference(q[..., nope:], cs)], -1)
        k = torch.cat([k_nope, apply_rope_reference(k_rope, cs)], -1)
        if self.use_qk_norm:
            q, k = self.q_norm(q), self.k_norm(k)
        v = v.contiguous()
        if ctx.cache is not None:
            o = ctx.cache.attend(self.layer_id, q, k, v)
        elif ctx.dense_mask is not None:
            o = _dense_attention(q, k, v, ctx.dense_mask)
        else:
            o = attention(q, k, v, causal=ctx.causal, seg=ctx.seg)
        o = o.reshape(B, S, H * D)
        if self.use_gated_attention:
            o = o * torch.sigmoid(self.gate(x))
        return self.o_proj(o, residual=residual)


__all__ = ["AttnContext", "AttnFactory", "GQA", "MLA", "attention_reference"]
