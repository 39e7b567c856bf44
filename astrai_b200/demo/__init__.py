"""Demos (parity: scripts/demo/*.py of the reference).

    python -m astrai_b200.demo.download --local-dir params      # fetch weights from the HF hub
    python -m astrai_b200.demo.chat --model_path params         # interactive streaming chat
    python -m astrai_b200.demo.batch --model_path params        # one batched, non-streaming call
    python -m astrai_b200.demo.generate --model_path params     # raw (no chat template) streaming

All of them load ``AutoModel`` / ``AutoTokenizer`` from a model directory in
bf16 on the GPU and talk to :class:`astrai_b200.inference.InferenceEngine`.
"""

from __future__ import annotations

from pathlib import Path

import torch

DEFAULT_PARAMS = Path.cwd() / "params"


def load_engine(model_path, max_batch_size: int = 1, device: str = "cuda"):
    from astrai_b200.inference import InferenceEngine
    from astrai_b200.models import AutoModel
    from astrai_b200.tokenize import AutoTokenizer

    model = AutoModel.from_pretrained(model_path)
    tok = AutoTokenizer.from_pretrained(model_path)
    dtype = torch.bfloat16 if device.startswith("cuda") else torch.float32
    model.to(device=device, dtype=dtype).eval()
    return InferenceEngine(model=model, tokenizer=tok, max_batch_size=max_batch_size), tok
