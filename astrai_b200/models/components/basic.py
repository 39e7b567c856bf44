"""Leaf modules: Linear, RMSNorm, Embedding (+NEFTune), RotaryEmbedding.

Parameter names, shapes and init follow the reference so checkpoints load
unchanged (astrai/model/components/{linear,norm,embedding,rope}.py):
Linear weight ``[out, in]`` ~ N(0, init_std), bias-free by default; RMSNorm
weight init 1; Embedding ~ N(0, 0.02); NEFTune adds Gaussian noise scaled by
``alpha / sqrt(seq_len)`` in training mode; RoPE keeps a non-persistent
``freqs_cis`` buffer of (cos, sin) pairs ``[max_len, dim/2, 2]``.
"""

from __future__ import annotations

import math
from typing import Dict, Optional

import torch
import torch.nn as nn

from astrai_b200.ops.embedding import embedding as _embedding
from astrai_b200.ops.gemm import linear as _linear
from astrai_b200.ops.gemm import packed_linear as _packed_linear
from astrai_b200.ops.norm import rms_norm as _rms_norm
from astrai_b200.ops.rope import ntk_base, rope_table


class Linear(nn.Module):
    def __init__(self, in_dim: int, out_dim: int, bias: bool = False, init_std: float = 0.02):
        super().__init__()
        self.weight = nn.Parameter(torch.empty((out_dim, in_dim)))
        self.bias = nn.Parameter(torch.zeros(out_dim)) if bias else None
        self.init_std = init_std
        self.reset_parameters()  # N(0, init_std) at construction, as the reference Linear

    @property
    def in_features(self) -> int:
        return self.weight.shape[1]

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def reset_parameters(self) -> None:
        nn.init.normal_(self.weight, mean=0.0, std=self.init_std)
        if self.bias is not None:
            bound = 1.0 / math.sqrt(self.weight.shape[1])
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.bias is None:
            return _packed_linear(x, [self.weight], residual=residual)
        return _linear(x, self.weight, residual=residual, bias=self.bias)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, norm_eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.normalized_shape = (dim,)
        self.norm_eps = norm_eps if norm_eps is not None else 1e-6

    def reset_parameters(self) -> None:
        nn.init.ones_(self.weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _rms_norm(x, self.weight, self.norm_eps)

    def forward_fork(self, x: torch.Tensor):
        """``(self(x), x)`` where the gradient of the second output is added inside the norm backward."""
        from astrai_b200.ops.norm import rms_norm_fork

        return rms_norm_fork(x, self.weight, self.norm_eps)


class Embedding(nn.Module):
    def __init__(self, vocab_size: int, embedding_dim: int, neftune_alpha: float = 0.0):
        super().__init__()
        self.weight = nn.Parameter(torch.empty((vocab_size, embedding_dim)))
        self.neftune_noise_alpha = neftune_alpha or 0.0

    def set_neftune_alpha(self, alpha: float) -> None:
        self.neftune_noise_alpha = alpha

    def reset_parameters(self) -> None:
        nn.init.normal_(self.weight, mean=0.0, std=0.02)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        out = _embedding(ids, self.weight)
        if self.training and self.neftune_noise_alpha > 0.0:
            eps = self.neftune_noise_alpha / math.sqrt(out.size(1))
            out = out + eps * torch.randn_like(out)
        return out


class RotaryEmbedding(nn.Module):
    """Interleaved RoPE angle table; stays fp32 when the model is cast."""

    def __init__(self, dim: int, max_len: int, base: float = 10000.0, rope_scaling: Optional[Dict] = None):
        super().__init__()
        self.dim = dim
        self.max_len = max_len or 4096
        self.base = base if base is not None else 10000.0
        self.rope_scaling = rope_scaling
        if rope_scaling is not None and rope_scaling.get("type", "ntk") == "ntk":
            self.base = ntk_base(self.base, dim, rope_scaling.get("factor", 1.0))
        self.register_buffer("freqs_cis", rope_table(dim, self.max_len, self.base), persistent=False)

    def _apply(self, fn, recurse=True):
        # keep the angle table in fp32 whatever dtype the model is cast to
        super()._apply(fn, recurse)
        if self.freqs_cis.dtype != torch.float32:
            self.freqs_cis = rope_table(self.dim, self.max_len, self.base, device=self.freqs_cis.device)
        return self

    def reset_buffers(self) -> None:
        """Recompute the angle table in place (after ``to_empty`` left it uninitialised)."""
        self.freqs_cis = rope_table(self.dim, self.max_len, self.base, device=self.freqs_cis.device)

    def table(self) -> torch.Tensor:
        return self.freqs_cis

    def forward(self, x: torch.Tensor, position_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        """(cos, sin) rows for the given positions: [B, S, dim/2, 2]."""
        if position_ids is None:
            return self.freqs_cis[: x.size(1)].unsqueeze(0).expand(x.size(0), -1, -1, -1)
        return self.freqs_cis[position_ids]
