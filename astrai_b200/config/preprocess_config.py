"""Declarative JSONL -> token preprocessing config (the ``dataset_config.json`` schema).

The schema is a file format shared with the reference
(astrai/config/preprocess_config.py:14-112): ``input.sections`` (single
output: SFT / pretraining) or ``input.sources`` (named outputs: DPO /
GRPO), a role -> ``train``/``mask`` map, ``preprocessing`` limits and packing,
and ``output`` storage / sharding / position-id mode.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

from astrai_b200.config.base import BaseConfig


@dataclass
class InputConfig(BaseConfig):
    sections: Optional[List[Dict]] = None
    sources: Optional[Dict[str, Dict]] = None


@dataclass
class ProcessingConfig(BaseConfig):
    max_seq_len: int = 2048
    min_chars: int = 50
    max_chars: int = 2_000_000
    max_items: Optional[int] = None
    batch_size: int = 256
    packing_strategy: str = "simple"    # simple | bfd | bfd_split
    max_packed_len: int = 8192
    truncation_mode: str = "keep_start"  # keep_start | keep_end


@dataclass
class OutputConfig(BaseConfig):
    domain_key: Optional[str] = None
    storage_format: str = "bin"          # bin | h5
    max_tokens_per_shard: int = 100_000_000
    dtype: Dict[str, str] = field(default_factory=dict)
    position_ids_mode: str = "doc_reset"  # none | doc_reset | continuous


@dataclass
class PipelineConfig(BaseConfig):
    version: int = 1
    input: InputConfig = field(default_factory=InputConfig)
    mask: Dict[str, str] = field(default_factory=dict)
    mask_default: str = "mask"
    preprocessing: ProcessingConfig = field(default_factory=ProcessingConfig)
    output: OutputConfig = field(default_factory=OutputConfig)
