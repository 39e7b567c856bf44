"""Sentence-embedding encoder, model type ``embedding``.

Behaviour kept from the reference (astrai/model/encoder.py:16-97), so encoder checkpoints load
in both frameworks: the decoder trunk of the LM without ``lm_head`` (a saved ``lm_head.weight``
is ignored on load), attention over the whole sequence with padding keys masked out, and one
vector per sequence pooled as ``cls`` (first position), ``last`` (last valid position) or
``mean`` (over valid positions; the default), optionally L2-normalised.

Here the trunk is the LM's own (:func:`build_trunk` / :func:`run_trunk`), and padding is
expressed as segment ids for the flash-attention kernel: valid tokens share segment 0 and every
padding position gets a segment of its own, so no valid query attends to padding.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, Mapping, Optional

import torch
import torch.nn.functional as F

from astrai_b200.config.model_config import EncoderConfig
from astrai_b200.models.automodel import AutoModel
from astrai_b200.models.components.attention import AttnContext
from astrai_b200.models.transformer import build_trunk, run_trunk


def _pool_cls(h: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    return h[:, 0]


def _pool_last(h: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    if mask is None:
        return h[:, -1]
    last = mask.long().sum(1) - 1
    return h[torch.arange(h.shape[0], device=h.device), last]


def _pool_mean(h: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
    if mask is None:
        return h.mean(1)
    w = mask.to(h.dtype).unsqueeze(-1)
    return (h * w).sum(1) / w.sum(1).clamp(min=1.0)


POOLERS: Dict[str, Callable[[torch.Tensor, Optional[torch.Tensor]], torch.Tensor]] = {
    "cls": _pool_cls, "last": _pool_last, "mean": _pool_mean,
}


def padding_segments(mask: torch.Tensor) -> torch.Tensor:
    """[B, S] validity mask -> segment ids: 0 for valid tokens, -(position + 1) for padding."""
    S = mask.shape[1]
    own = -torch.arange(1, S + 1, device=mask.device, dtype=torch.int32)
    return torch.where(mask.bool(), torch.zeros_like(own), own).expand_as(mask).contiguous()


@AutoModel.register("embedding")
class EmbeddingEncoder(AutoModel):
    def __init__(self, config: EncoderConfig):
        super().__init__(config)
        build_trunk(self, config)
        self.pooling_type = config.pooling_type or "mean"
        if self.pooling_type not in POOLERS:
            raise ValueError(f"pooling_type {self.pooling_type!r}: choose one of {sorted(POOLERS)}")
        self.normalize_embeddings = bool(config.normalize_embeddings)
        for m in self.modules():
            if m is not self and hasattr(m, "reset_parameters"):
                m.reset_parameters()

    def load_state_dict(self, state_dict: Mapping[str, Any], strict: bool = True, assign: bool = False):
        return super().load_state_dict({k: v for k, v in state_dict.items() if k != "lm_head.weight"},
                                       strict=strict, assign=assign)

    def forward(self, input_ids: torch.Tensor, input_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S = input_ids.shape
        seg = padding_segments(input_mask) if input_mask is not None else None
        ctx = AttnContext(B=B, S=S, table=self.rotary_embedding.table(), positions=position_ids, seg=seg,
                          causal=False)
        pooled = POOLERS[self.pooling_type](run_trunk(self, input_ids, ctx), input_mask)
        return F.normalize(pooled, p=2, dim=-1) if self.normalize_embeddings else pooled
