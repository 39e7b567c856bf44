"""OpenAI / Anthropic compatible server.

    python -m astrai_b200.cli.server --param_path MODEL_DIR [--host 0.0.0.0] [--port 8000] [--max_batch_size 16]

Parity: scripts/tools/server.py:9-68 of the reference (same flags). Added:
``--n_pages`` / ``--page_size`` serve from a paged KV cache with prefix
sharing instead of the per-slot cache.
"""

from __future__ import annotations

import argparse
from pathlib import Path
from typing import List, Optional

import torch


def main(argv: Optional[List[str]] = None) -> None:
    from astrai_b200.inference.api.server import run_server

    p = argparse.ArgumentParser(description="Start the AstrAI-B200 inference server.")
    p.add_argument("--host", default="0.0.0.0")
    p.add_argument("--port", type=int, default=8000)
    p.add_argument("--reload", action="store_true")
    p.add_argument("--param_path", default=None, help="Model directory (config.json, weights, tokenizer).")
    p.add_argument("--device", type=str, default="cuda")
    p.add_argument("--dtype", type=str, default="bfloat16", choices=["bfloat16", "float16", "float32"])
    p.add_argument("--max_batch_size", type=int, default=16)
    p.add_argument("--n_pages", type=int, default=None, help="Paged KV cache with this many pages.")
    p.add_argument("--page_size", type=int, default=128)
    a = p.parse_args(argv)
    if a.param_path is None:
        raise SystemExit("--param_path is required")
    dtype = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[a.dtype]
    extra = {"n_pages": a.n_pages, "page_size": a.page_size} if a.n_pages else {}
    run_server(Path(a.param_path), host=a.host, port=a.port, reload=a.reload, device=a.device, dtype=dtype,
               max_batch_size=a.max_batch_size, **extra)


if __name__ == "__main__":
    main()
