"""Raw autoregressive streaming (parity: scripts/demo/generate_ar.py of the reference): the
prompt goes to the model as-is, without a chat template."""

from __future__ import annotations

import argparse
from pathlib import Path

from astrai_b200.demo import DEFAULT_PARAMS, load_engine


def generate_text(argv=None, prompt=None, engine=None):
    p = argparse.ArgumentParser(description="Raw streaming generation")
    p.add_argument("--model_path", type=Path, default=DEFAULT_PARAMS)
    p.add_argument("--max_tokens", type=int, default=2048)
    p.add_argument("--device", type=str, default="cuda")
    a = p.parse_args(argv)
    if engine is None:
        engine, _ = load_engine(a.model_path, device=a.device)
    query = prompt if prompt is not None else input(">> ")
    out = ""
    for piece in engine.generate(prompt=query, stream=True, max_tokens=a.max_tokens, temperature=0.8, top_p=0.95,
                                 top_k=50):
        print(piece, end="", flush=True)
        out += piece
    print()
    return out


if __name__ == "__main__":
    generate_text()
