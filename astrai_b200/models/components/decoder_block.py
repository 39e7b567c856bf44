"""Pre-norm decoder block (parity: astrai/model/components/decoder_block.py:13-49).

``x = x + attn(input_norm(x)); x = x + ffn(post_attention_norm(x))`` with the
module names ``attention``, ``input_norm``, ``post_attention_norm``, ``mlp``.
Both residual adds happen inside the output-projection GEMM epilogues.
``first_k_dense`` (a config addition) makes the first k layers of an MoE
model use the dense MLP.
"""

from __future__ import annotations

from dataclasses import asdict

import torch
import torch.nn as nn

from astrai_b200.models.components.attention import AttnContext, AttnFactory
from astrai_b200.models.components.basic import RMSNorm
from astrai_b200.models.components.mlp import FFNFactory


class DecoderBlock(nn.Module):
    def __init__(self, config, layer_id: int):
        super().__init__()
        cfg = asdict(config)
        cfg.update(
            dim=config.hidden_size,
            dim_ffn=config.intermediate_size,
            n_layers=config.num_hidden_layers,
            n_heads=config.num_attention_heads,
            n_kv_heads=config.num_key_value_heads or config.num_attention_heads,
            norm_eps=config.rms_norm_eps,
            down_init_std=0.02 / (2 * config.num_hidden_layers) ** 0.5,
        )
        self.layer_id = layer_id
        self.attention = AttnFactory.create(config.attn_type or "gqa", **cfg, layer_id=layer_id)
        self.input_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        ffn_type = config.ffn_type or "mlp"
        first_dense = getattr(config, "first_k_dense", None) or 0
        if ffn_type == "moe" and layer_id < first_dense:
            ffn_type = "mlp"
        self.mlp = FFNFactory.create(ffn_type, **cfg)

    def forward(self, x: torch.Tensor, ctx: AttnContext) -> torch.Tensor:
        # forward_fork: the residual branch's gradient is summed inside the norm backward kernel
        xn, xr = self.input_norm.forward_fork(x)
        h = self.attention(xn, ctx, residual=xr)
        hn, hr = self.post_attention_norm.forward_fork(h)
        return self.mlp(hn, residual=hr, ctx=ctx)
