from astrai_b200.models.automodel import AutoModel
from astrai_b200.models.components import (
    GQA, MLA, MLP, AttnFactory, DecoderBlock, DeepSeekMoE, Embedding, FFNFactory, Linear, LoRAConfig, LoRALinear,
    RMSNorm, RotaryEmbedding, inject_lora, load_lora, merge_lora, save_lora,
)
from astrai_b200.models.encoder import EmbeddingEncoder
from astrai_b200.models.transformer import AutoRegressiveLM

__all__ = [
    "AutoModel", "AutoRegressiveLM", "EmbeddingEncoder", "Linear", "RMSNorm", "MLP", "GQA", "MLA", "DeepSeekMoE",
    "DecoderBlock", "Embedding", "RotaryEmbedding", "AttnFactory", "FFNFactory", "LoRAConfig", "LoRALinear",
    "inject_lora", "merge_lora", "save_lora", "load_lora",
]
