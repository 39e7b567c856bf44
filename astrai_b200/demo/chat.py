"""Interactive streaming chat (parity: scripts/demo/stream_chat.py of the reference).

Type a message; ``!exit`` quits. Every turn is a fresh single-turn chat (as in
the reference), streamed token by token with the frequency penalty applied
over the last ``--rep_window`` tokens.
"""

from __future__ import annotations

import argparse
from pathlib import Path
from typing import Iterable, Optional

from astrai_b200.demo import DEFAULT_PARAMS, load_engine


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="Interactive streaming chat")
    p.add_argument("--model_path", type=Path, default=DEFAULT_PARAMS)
    p.add_argument("--temperature", type=float, default=0.8)
    p.add_argument("--top_p", type=float, default=0.95)
    p.add_argument("--top_k", type=int, default=50)
    p.add_argument("--max_tokens", type=int, default=2048)
    p.add_argument("--frequency_penalty", type=float, default=0.5)
    p.add_argument("--rep_window", type=int, default=64)
    p.add_argument("--system_prompt", type=str, default="")
    p.add_argument("--device", type=str, default="cuda")
    return p.parse_args(argv)


def chat(argv=None, queries: Optional[Iterable[str]] = None, engine=None, tokenizer=None) -> list:
    a = parse_args(argv)
    if engine is None:
        engine, tokenizer = load_engine(a.model_path, device=a.device)
    src = iter(queries) if queries is not None else iter(lambda: input(">> "), None)
    replies = []
    for q in src:
        if q == "!exit":
            break
        msgs = ([{"role": "system", "content": a.system_prompt}] if a.system_prompt else [])
        msgs.append({"role": "user", "content": q})
        prompt = tokenizer.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True)
        out = ""
        for piece in engine.generate(prompt=prompt, stream=True, max_tokens=a.max_tokens, temperature=a.temperature,
                                     top_p=a.top_p, top_k=a.top_k, frequency_penalty=a.frequency_penalty,
                                     rep_window=a.rep_window):
            print(piece, end="", flush=True)
            out += piece
        print()
        replies.append(out)
    return replies


if __name__ == "__main__":
    chat()
