"""Autoregressive decoder LM (parity: astrai/model/transformer.py:17-122).

Embedding -> N x DecoderBlock -> RMSNorm -> lm_head; returns
``{"logits", "hidden_states"}``. Tied embeddings share one tensor; the tied
``lm_head.weight`` is dropped from ``state_dict()`` and re-aliased on load,
exactly as the reference does, so checkpoints are interchangeable.

Attention masking: with no mask the attention is causal. ``seg_ids`` ([B, S]
int; query q sees key k only if equal) is the fast path used by the
framework's own strategies for packed documents and padding. A dense
``input_mask`` (2-D key mask, 3-D or 4-D boolean, reference semantics: no
implicit causality) takes the generic path.
"""

from __future__ import annotations

from typing import Any, Dict, Mapping, Optional

import torch
import torch.nn as nn

from astrai_b200.config.model_config import AutoRegressiveLMConfig
from astrai_b200.models.automodel import AutoModel
from astrai_b200.models.components.attention import AttnContext
from astrai_b200.models.components.basic import Embedding, Linear, RMSNorm, RotaryEmbedding
from astrai_b200.models.components.decoder_block import DecoderBlock


def process_attention_mask(input_mask: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if input_mask is None:
        return None
    if input_mask.dim() == 2:
        return input_mask[:, None, None, :]
    if input_mask.dim() == 3:
        return input_mask[:, None, :, :]
    return input_mask


def _rope_dim(config) -> int:
    if getattr(config, "attn_type", "gqa") == "mla":
        return config.qk_rope_head_dim
    return config.hidden_size // config.num_attention_heads


def build_trunk(model: nn.Module, config) -> None:
    """The decoder stack shared by the LM and the embedding encoder, under the attribute names that
    are the checkpoint keys: ``rotary_embedding`` (angle table, base 10000 when the config has
    none), ``embed_tokens``, ``layers`` and the final ``norm``."""
    base = config.rope_theta if config.rope_theta is not None else 10000
    model.rotary_embedding = RotaryEmbedding(_rope_dim(config), config.max_position_embeddings, base,
                                             rope_scaling=config.rope_scaling)
    model.embed_tokens = Embedding(config.vocab_size, config.hidden_size, neftune_alpha=config.neftune_alpha)
    model.layers = nn.ModuleList([DecoderBlock(config, i) for i in range(config.num_hidden_layers)])
    model.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)


def run_trunk(model: nn.Module, input_ids: torch.Tensor, ctx: AttnContext) -> torch.Tensor:
    x = model.embed_tokens(input_ids)
    for layer in model.layers:
        x = layer(x, ctx)
    return model.norm(x)


@AutoModel.register("autoregressive_lm")
class AutoRegressiveLM(AutoModel):
    def __init__(self, config: AutoRegressiveLMConfig):
        super().__init__(config)
        build_trunk(self, config)
        self.lm_head = Linear(config.hidden_size, config.vocab_size)
        if config.tie_word_embeddings is True:
            self.lm_head.weight = self.embed_tokens.weight
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module):
        if hasattr(module, "reset_parameters") and not isinstance(module, AutoModel):
            module.reset_parameters()

    def tied_parameters(self):
        return [("lm_head.weight", "embed_tokens.weight")] if self.config.tie_word_embeddings is True else []

    # ------------------------------------------------------------------ state dict (tied lm_head)
    def load_state_dict(self, state_dict: Mapping[str, Any], strict: bool = True, assign: bool = False):
        sd = dict(state_dict)
        if self.config.tie_word_embeddings is True:
            if "embed_tokens.weight" in sd:
                sd["lm_head.weight"] = sd["embed_tokens.weight"]
        elif "lm_head.weight" not in sd and "embed_tokens.weight" in sd:
            sd["lm_head.weight"] = sd["embed_tokens.weight"].clone()
        return super().load_state_dict(sd, strict, assign)

    def state_dict(self, destination=None, prefix="", keep_vars=False):
        sd = super().state_dict(destination=destination, prefix=prefix, keep_vars=keep_vars)
        if self.config.tie_word_embeddings is True:
            sd.pop(prefix + "lm_head.weight", None)
        return sd

    # ------------------------------------------------------------------ forward
    def make_context(self, input_ids, input_mask=None, paged_cache=None, position_ids=None, seg_ids=None):
        B, S = input_ids.shape
        mask = process_attention_mask(input_mask)
        return AttnContext(B=B, S=S, table=self.rotary_embedding.table(), positions=position_ids, seg=seg_ids,
                           dense_mask=mask, causal=mask is None, cache=paged_cache,
                           aux_losses=[] if self.training else None)

    def backbone(self, input_ids: torch.Tensor, ctx: AttnContext) -> torch.Tensor:
        return run_trunk(self, input_ids, ctx)

    def forward(self, input_ids: torch.Tensor, input_mask: Optional[torch.Tensor] = None, paged_cache=None,
                position_ids: Optional[torch.Tensor] = None, seg_ids: Optional[torch.Tensor] = None,
                logits_to_keep=None) -> Dict[str, torch.Tensor]:
        """``logits_to_keep``: None (all positions), an int n (the last n positions), or a bool
        ``[B, S]`` tensor selecting positions, in which case ``logits`` is ``[N, V]`` in row-major
        order of the selected positions (scoring packed documents without full-vocab logits)."""
        assert input_ids.ndim == 2
        ctx = self.make_context(input_ids, input_mask, paged_cache, position_ids, seg_ids)
        hidden = self.backbone(input_ids, ctx)
        if isinstance(logits_to_keep, torch.Tensor):
            h = hidden[logits_to_keep]  # bool [B, S]: logits [N, V] for the selected positions only
        else:
            h = hidden if logits_to_keep is None else hidden[:, -logits_to_keep:]
        out = {"logits": self.lm_head(h), "hidden_states": hidden}
        if ctx.aux_losses:
            out["aux_loss"] = torch.stack(ctx.aux_losses).sum()
        return out
