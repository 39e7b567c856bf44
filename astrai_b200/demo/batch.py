"""Batched chat generation (parity: scripts/demo/generate_batch.py of the reference): several
chat prompts in one non-streaming ``generate`` call; the engine decodes them together."""

from __future__ import annotations

import argparse
from pathlib import Path

from astrai_b200.demo import DEFAULT_PARAMS, load_engine

QUERIES = ["Hello", "What is artificial intelligence?", "How is the weather today?",
           "I feel anxious, what should I do?", "What is a graphics card?"]


def batch_generate(argv=None, engine=None, tokenizer=None):
    p = argparse.ArgumentParser(description="Batched chat generation")
    p.add_argument("--model_path", type=Path, default=DEFAULT_PARAMS)
    p.add_argument("--max_tokens", type=int, default=2048)
    p.add_argument("--queries", type=str, nargs="*", default=QUERIES)
    p.add_argument("--device", type=str, default="cuda")
    a = p.parse_args(argv)
    if engine is None:
        engine, tokenizer = load_engine(a.model_path, max_batch_size=len(a.queries), device=a.device)
    prompts = [tokenizer.apply_chat_template([{"role": "user", "content": q}], tokenize=False,
                                             add_generation_prompt=True) for q in a.queries]
    outs = engine.generate(prompt=prompts, stream=False, max_tokens=a.max_tokens, temperature=0.8, top_p=0.95,
                           top_k=50)
    for q, r in zip(a.queries, outs):
        print((q, r))
    return outs


if __name__ == "__main__":
    batch_generate()
