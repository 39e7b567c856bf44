"""Model configs (the ``config.json`` of a model directory).

The field names are the on-disk interface shared with the reference
(astrai/config/model_config.py:26-82) so that model directories are
interchangeable. Additions of this framework, all optional and defaulting to
the reference behaviour:

* ``first_k_dense``      - the first k layers use the dense SwiGLU MLP even
                            when ``ffn_type == "moe"``;
* ``moe_intermediate_size`` - FFN width of each expert (defaults to
                            ``intermediate_size``);
* ``moe_aux_loss_coef``  - coefficient of the switch-style balance loss;
* ``shared_expert_mode`` - ``"mean"`` (reference: shared experts averaged)
                            or ``"sum"``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Optional

from astrai_b200.config.base import BaseConfig
from astrai_b200.factory import Registry


class ConfigFactory(Registry[BaseConfig]):
    """Picks the config class from the ``model_type`` key."""

    @classmethod
    def load(cls, raw: Dict[str, Any]) -> BaseConfig:
        kind = raw.get("model_type") or "autoregressive_lm"
        return cls.get_component_class(kind).from_dict(raw)


@dataclass
class BaseModelConfig(BaseConfig):
    model_type: Optional[str] = None
    neftune_alpha: float = 0.0


@ConfigFactory.register("autoregressive_lm")
@dataclass
class AutoRegressiveLMConfig(BaseModelConfig):
    vocab_size: Optional[int] = None
    hidden_size: Optional[int] = None
    num_hidden_layers: Optional[int] = None
    rms_norm_eps: Optional[float] = None
    intermediate_size: Optional[int] = None
    tie_word_embeddings: Optional[bool] = None
    max_position_embeddings: Optional[int] = None
    rope_theta: Optional[float] = None
    rope_scaling: Optional[dict] = None
    attn_type: str = "gqa"
    num_attention_heads: Optional[int] = None
    num_key_value_heads: Optional[int] = None
    use_qk_norm: Optional[bool] = None
    use_gated_attention: Optional[bool] = None
    kv_lora_rank: Optional[int] = None
    qk_nope_head_dim: Optional[int] = None
    qk_rope_head_dim: Optional[int] = None
    ffn_type: str = "mlp"
    n_routed_experts: Optional[int] = None
    n_shared_experts: Optional[int] = None
    n_activated_experts: Optional[int] = None
    topk_method: Optional[str] = None
    # framework additions (absent keys keep reference semantics)
    first_k_dense: Optional[int] = None
    moe_intermediate_size: Optional[int] = None
    moe_aux_loss_coef: Optional[float] = None
    shared_expert_mode: Optional[str] = None


@ConfigFactory.register("embedding")
@dataclass
class EncoderConfig(BaseModelConfig):
    # saved into config.json, so AutoModel.from_pretrained rebuilds an encoder, not an LM
    model_type: Optional[str] = "embedding"
    vocab_size: Optional[int] = None
    hidden_size: Optional[int] = None
    num_hidden_layers: Optional[int] = None
    rms_norm_eps: Optional[float] = None
    intermediate_size: Optional[int] = None
    max_position_embeddings: Optional[int] = None
    rope_theta: Optional[float] = None
    rope_scaling: Optional[dict] = None
    attn_type: str = "gqa"
    num_attention_heads: Optional[int] = None
    num_key_value_heads: Optional[int] = None
    use_qk_norm: Optional[bool] = None
    use_gated_attention: Optional[bool] = None
    ffn_type: str = "mlp"
    pooling_type: Optional[str] = None
    normalize_embeddings: Optional[bool] = None
