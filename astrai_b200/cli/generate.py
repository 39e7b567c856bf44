"""Batch generation from a JSONL file.

    python -m astrai_b200.cli.generate --param_path MODEL_DIR --input_json_file in.jsonl --output_json_file out.jsonl

Parity: scripts/tools/generate.py:15-215 of the reference (same flags and
defaults; rows with ``messages`` go through the chat template and keep their
fields, others use ``--question_key``; ``--num_samples`` repeats each prompt).
"""

from __future__ import annotations

import argparse
import json
import time
from typing import List, Optional

import torch


def main(argv: Optional[List[str]] = None) -> None:
    from astrai_b200.inference import InferenceEngine
    from astrai_b200.models import AutoModel
    from astrai_b200.tokenize import AutoTokenizer

    p = argparse.ArgumentParser(description="Batch generation from JSONL file.")
    p.add_argument("--param_path", type=str, required=True)
    p.add_argument("--input_json_file", type=str, required=True)
    p.add_argument("--output_json_file", type=str, required=True)
    p.add_argument("--question_key", type=str, default="question")
    p.add_argument("--response_key", type=str, default="response")
    p.add_argument("--temperature", type=float, default=0.60)
    p.add_argument("--top_k", type=int, default=30)
    p.add_argument("--top_p", type=float, default=0.95)
    p.add_argument("--batch_size", type=int, default=1)
    p.add_argument("--num_samples", type=int, default=1)
    p.add_argument("--max_tokens", type=int, default=None)
    p.add_argument("--cache_len", type=int, default=2048)
    p.add_argument("--frequency_penalty", type=float, default=0.0)
    p.add_argument("--rep_window", type=int, default=64)
    a = p.parse_args(argv)
    t0 = time.time()
    model = AutoModel.from_pretrained(a.param_path).to(device="cuda", dtype=torch.bfloat16).eval()
    tok = AutoTokenizer.from_pretrained(a.param_path)
    rows = [json.loads(line) for line in open(a.input_json_file, encoding="utf-8") if line.strip()]
    chat = bool(rows) and "messages" in rows[0]
    prompts = [tok.apply_chat_template(r["messages"], tokenize=False) if chat else r[a.question_key] for r in rows]
    max_tokens = a.max_tokens or model.config.max_position_embeddings
    n = max(1, a.batch_size)
    with InferenceEngine(model, tok, max_batch_size=n * a.num_samples, max_seq_len=a.cache_len,
                         max_prompt_len=a.cache_len) as eng, open(a.output_json_file, "w", encoding="utf-8") as out:
        for i in range(0, len(prompts), n):
            chunk = prompts[i:i + n]
            flat = [q for q in chunk for _ in range(a.num_samples)]
            res = eng.generate(flat, max_tokens=max_tokens, temperature=a.temperature, top_p=a.top_p, top_k=a.top_k,
                               frequency_penalty=a.frequency_penalty, rep_window=a.rep_window)
            for j, q in enumerate(chunk):
                r = res[j * a.num_samples:(j + 1) * a.num_samples]
                r = r if a.num_samples > 1 else r[0]
                item = {**rows[i + j], a.response_key: r} if chat else {a.question_key: q, a.response_key: r}
                out.write(json.dumps(item, ensure_ascii=False) + "\n")
    dt = time.time() - t0
    print(f"Done: {len(prompts)} prompts x {a.num_samples} samples -> {a.output_json_file} in {dt:.1f}s")


if __name__ == "__main__":
    main()
