from astrai_b200.models.components.attention import GQA, MLA, AttnContext, AttnFactory
from astrai_b200.models.components.basic import Embedding, Linear, RMSNorm, RotaryEmbedding
from astrai_b200.models.components.decoder_block import DecoderBlock
from astrai_b200.models.components.lora import (
    LoRAConfig,
    LoRALinear,
    inject_lora,
    load_lora,
    merge_lora,
    save_lora,
)
from astrai_b200.models.components.mlp import MLP, DeepSeekMoE, FFNFactory

__all__ = [
    "GQA", "MLA", "AttnContext", "AttnFactory", "Embedding", "Linear", "RMSNorm", "RotaryEmbedding",
    "DecoderBlock", "LoRAConfig", "LoRALinear", "inject_lora", "load_lora", "merge_lora", "save_lora",
    "MLP", "DeepSeekMoE", "FFNFactory",
]
