"""Shared helpers of the evaluation suite: input discovery, model loading, statistics."""

from __future__ import annotations

import glob
import json
import os
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch


def collect_input_files(path: str) -> List[str]:
    """A directory (every ``*.jsonl`` / ``*.json`` below it), a glob, or one file."""
    if os.path.isdir(path):
        found = glob.glob(os.path.join(path, "**", "*.jsonl"), recursive=True)
        found += glob.glob(os.path.join(path, "**", "*.json"), recursive=True)
        return sorted(found)
    return sorted(glob.glob(path))


def load_items(path: str) -> List[dict]:
    """JSONL (one object per line) or JSON (an array or a single object)."""
    with open(path, encoding="utf-8") as fh:
        if path.lower().endswith(".json"):
            data = json.load(fh)
            return [data] if isinstance(data, dict) else list(data)
        return [json.loads(line) for line in fh if line.strip()]


def default_device() -> str:
    return "cuda" if torch.cuda.is_available() else "cpu"


def default_dtype() -> str:
    return "bfloat16" if torch.cuda.is_available() else "float32"


def load_model(param_path: str, device: Optional[str] = None, dtype: Optional[str] = None):
    """(model, tokenizer) from a model directory, in eval mode on ``device`` / ``dtype``."""
    from astrai_b200.models import AutoModel
    from astrai_b200.tokenize import AutoTokenizer

    model = AutoModel.from_pretrained(param_path)
    model.to(device=device or default_device(), dtype=getattr(torch, dtype or default_dtype())).eval()
    return model, AutoTokenizer.from_pretrained(param_path)


def percentiles(values: Sequence[float], qs=(50, 90, 95, 99)) -> Dict[str, float]:
    """Linearly interpolated percentiles (numpy's default rule) as ``{"p50": ...}``."""
    if len(values) == 0:
        return {}
    arr = np.asarray(values, dtype=np.float64)
    return {f"p{q}": float(np.percentile(arr, q)) for q in qs}


def write_json(path: Optional[str], data) -> None:
    if path:
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        with open(path, "w", encoding="utf-8") as fh:
            json.dump(data, fh, ensure_ascii=False, indent=2)
