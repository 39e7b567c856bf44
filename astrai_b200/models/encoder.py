"""Embedding encoder (parity: astrai/model/encoder.py:16-97).

Same trunk as the LM without ``lm_head``; bidirectional attention (a 2-D
key mask marks padding); pooling ``cls`` / ``last`` / ``mean`` (masked);
optional L2 normalisation. Registered as model type ``embedding``.
"""

from __future__ import annotations

from typing import Any, Mapping, Optional

import torch
import torch.nn as nn

from astrai_b200.config.model_config import EncoderConfig
from astrai_b200.models.automodel import AutoModel
from astrai_b200.models.components.attention import AttnContext
from astrai_b200.models.components.basic import Embedding, RMSNorm, RotaryEmbedding
from astrai_b200.models.components.decoder_block import DecoderBlock


@AutoModel.register("embedding")
class EmbeddingEncoder(AutoModel):
    def __init__(self, config: EncoderConfig):
        super().__init__(config)
        self.rotary_embedding = RotaryEmbedding(config.hidden_size // config.num_attention_heads,
                                                config.max_position_embeddings,
                                                config.rope_theta if config.rope_theta is not None else 10000,
                                                rope_scaling=config.rope_scaling)
        self.embed_tokens = Embedding(config.vocab_size, config.hidden_size, neftune_alpha=config.neftune_alpha)
        self.layers = nn.ModuleList([DecoderBlock(config, i) for i in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.pooling_type = config.pooling_type or "mean"
        self.normalize_embeddings = bool(config.normalize_embeddings)
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module):
        if hasattr(module, "reset_parameters") and not isinstance(module, AutoModel):
            module.reset_parameters()

    def load_state_dict(self, state_dict: Mapping[str, Any], strict: bool = True, assign: bool = False):
        sd = dict(state_dict)
        sd.pop("lm_head.weight", None)
        return super().load_state_dict(sd, strict=strict, assign=assign)

    def forward(self, input_ids: torch.Tensor, input_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S = input_ids.shape
        # bidirectional; padding keys get unique negative segment ids
        seg = None
        if input_mask is not None:
            valid = input_mask.bool()
            pad_id = -(torch.arange(S, device=input_ids.device, dtype=torch.int32) + 1).expand(B, S)
            seg = torch.where(valid, torch.zeros_like(pad_id), pad_id)
        ctx = AttnContext(B=B, S=S, table=self.rotary_embedding.table(), positions=position_ids, seg=seg,
                          causal=False)
        x = self.embed_tokens(input_ids)
        for layer in self.layers:
            x = layer(x, ctx)
        h = self.norm(x)
        if self.pooling_type == "cls":
            pooled = h[:, 0]
        elif self.pooling_type == "last":
            if input_mask is not None:
                lengths = input_mask.long().sum(1) - 1
                pooled = h[torch.arange(B, device=h.device), lengths]
            else:
                pooled = h[:, -1]
        else:
            if input_mask is not None:
                m = input_mask.unsqueeze(-1).to(h.dtype)
                pooled = (h * m).sum(1) / m.sum(1).clamp(min=1.0)
            else:
                pooled = h.mean(1)
        if self.normalize_embeddings:
            pooled = torch.nn.functional.normalize(pooled, p=2, dim=-1)
        return pooled
