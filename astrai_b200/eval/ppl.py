"""Perplexity and token-level loss on JSONL / JSON text.

    python -m astrai_b200.eval.ppl --param_path MODEL --input_path DATA --output_dir OUT
        [--text_key text] [--batch_size 4] [--max_length 2048] [--token_level] [--max_samples N]

Parity: scripts/eval/evaluate_ppl.py of the reference: the same flags, a
``summary.json`` keyed by file label with ``overall`` (num_tokens, mean_loss,
ppl, median_loss, p50/p90/p95/p99) and, with ``--token_level``, per-record
``{label}_tokens.jsonl`` and a ``by_token_type`` breakdown (special / cjk /
non_ascii / ascii). Texts are truncated to ``max_length`` tokens; the first
token of each text is context only.

Execution differs: texts are packed best-fit-decreasing into rows through
:mod:`astrai_b200.eval.loglik` (``--batch_size`` x ``--max_length`` tokens per
forward), so short texts do not pay for padding, and every token's loss is
kept (4 bytes each) so percentiles are exact.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
from typing import Dict, List, Optional

import numpy as np

from astrai_b200.eval.common import (collect_input_files, default_device, default_dtype, load_items, load_model,
                                     percentiles, write_json)
from astrai_b200.eval.loglik import Doc, score_docs


def token_type(token_id: int, special: frozenset, decode) -> str:
    if token_id in special:
        return "special"
    text = decode([token_id], skip_special_tokens=True)
    if any("一" <= ch <= "鿿" for ch in text):
        return "cjk"
    if any(ord(ch) > 127 for ch in text):
        return "non_ascii"
    return "ascii"


def _summary(losses: np.ndarray) -> Dict:
    if losses.size == 0:
        return {}
    mean = float(losses.mean())
    out = {"num_tokens": int(losses.size), "mean_loss": mean, "ppl": math.exp(mean),
           "median_loss": float(np.median(losses))}
    out.update(percentiles(losses))
    return out


def evaluate_texts(model, tokenizer, texts: List[str], max_length: int = 2048, batch_size: int = 4,
                   token_level: bool = False) -> Dict:
    """Statistics (and per-record token rows when ``token_level``) for a list of texts."""
    ids = [tokenizer.encode(t)[:max_length] for t in texts]
    keep = [i for i, x in enumerate(ids) if len(x) >= 2]
    lps = score_docs(model, [Doc(ids[i], 1) for i in keep], max_len=max_length,
                     max_tokens=batch_size * max_length)
    losses = np.concatenate([-lp.numpy() for lp in lps]) if lps else np.zeros(0, np.float32)
    stats: Dict = {"overall": _summary(losses)} if losses.size else {}
    records = []
    if token_level and lps:
        special = frozenset(tokenizer.stop_ids)
        typed: Dict[str, List[float]] = {}
        for i, lp in zip(keep, lps):
            tok = ids[i][1:]
            lv = (-lp).tolist()
            for t, l in zip(tok, lv):
                typed.setdefault(token_type(t, special, tokenizer.decode), []).append(l)
            records.append({"text": texts[i][:200], "token_ids": tok, "log_probs": [round(-l, 4) for l in lv],
                            "ppl": math.exp(sum(lv) / len(lv)) if lv else None})
        stats["by_token_type"] = {k: _summary(np.asarray(v, np.float32)) for k, v in sorted(typed.items())}
    if records:
        stats["_records"] = records
    return stats


def run(param_path: str, input_path: str, output_dir: str, text_key: str = "text", batch_size: int = 4,
        max_length: int = 2048, token_level: bool = False, max_samples: Optional[int] = None,
        device: Optional[str] = None, dtype: Optional[str] = None, model=None, tokenizer=None) -> Dict:
    if model is None:
        model, tokenizer = load_model(param_path, device, dtype)
    files = collect_input_files(input_path)
    os.makedirs(output_dir, exist_ok=True)
    summary = {}
    for path in files:
        label = os.path.splitext(os.path.basename(path))[0]
        items = load_items(path)
        if max_samples and len(items) > max_samples:
            items = random.sample(items, max_samples)
        texts = [it[text_key] for it in items if text_key in it]
        if not texts:
            continue
        stats = evaluate_texts(model, tokenizer, texts, max_length, batch_size, token_level)
        records = stats.pop("_records", None)
        if records is not None:
            with open(os.path.join(output_dir, f"{label}_tokens.jsonl"), "w", encoding="utf-8") as fh:
                for r in records:
                    fh.write(json.dumps(r, ensure_ascii=False) + "\n")
        summary[label] = stats
        o = stats.get("overall", {})
        if o:
            print(f"[{label}] tokens={o['num_tokens']} loss={o['mean_loss']:.4f} ppl={o['ppl']:.3f}")
    write_json(os.path.join(output_dir, "summary.json"), summary)
    return summary


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Perplexity and token-level loss evaluation on JSONL/JSON data.")
    p.add_argument("--param_path", type=str, required=True)
    p.add_argument("--input_path", type=str, required=True)
    p.add_argument("--output_dir", type=str, required=True)
    p.add_argument("--text_key", type=str, default="text")
    p.add_argument("--batch_size", type=int, default=4)
    p.add_argument("--max_length", type=int, default=2048)
    p.add_argument("--token_level", action="store_true")
    p.add_argument("--max_samples", type=int, default=None)
    p.add_argument("--device", type=str, default=default_device())
    p.add_argument("--dtype", type=str, default=default_dtype())
    a = p.parse_args(argv)
    run(a.param_path, a.input_path, a.output_dir, a.text_key, a.batch_size, a.max_length, a.token_level,
        a.max_samples, a.device, a.dtype)


if __name__ == "__main__":
    main()
