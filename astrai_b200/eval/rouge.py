"""ROUGE-N and ROUGE-L (Lin, 2004) between reference and candidate texts.

    python -m astrai_b200.eval.rouge --data_path pairs.jsonl [--output scores.json]

Parity: scripts/eval/evaluate_rouge.py of the reference: JSONL rows with
``reference`` and ``candidate``; per-item scores and the mean precision /
recall / F1 of rouge-1, rouge-2 and rouge-l. Tokens are whitespace-separated
words, case kept (as the reference scores them); ROUGE-L uses the longest
common subsequence (O(n*m) dynamic programme kept to one row).
"""

from __future__ import annotations

import argparse
import json
from collections import Counter
from typing import Dict, List

from astrai_b200.eval.common import write_json

def tokenize(text: str) -> List[str]:
    return text.split()


def _prf(overlap: float, n_cand: int, n_ref: int) -> Dict[str, float]:
    p = overlap / n_cand if n_cand else 0.0
    r = overlap / n_ref if n_ref else 0.0
    return {"precision": p, "recall": r, "f1": 2 * p * r / (p + r) if p + r > 0 else 0.0}


def rouge_n(ref: List[str], cand: List[str], n: int) -> Dict[str, float]:
    rc = Counter(tuple(ref[i:i + n]) for i in range(len(ref) - n + 1))
    cc = Counter(tuple(cand[i:i + n]) for i in range(len(cand) - n + 1))
    return _prf(sum((rc & cc).values()), sum(cc.values()), sum(rc.values()))


def lcs_len(a: List[str], b: List[str]) -> int:
    if len(a) < len(b):
        a, b = b, a
    prev = [0] * (len(b) + 1)
    for x in a:
        cur = [0]
        for j, y in enumerate(b):
            cur.append(prev[j] + 1 if x == y else max(prev[j + 1], cur[j]))
        prev = cur
    return prev[-1]


def rouge_l(ref: List[str], cand: List[str]) -> Dict[str, float]:
    return _prf(lcs_len(ref, cand), len(cand), len(ref))


def compute_rouge(reference: str, candidate: str, n: int = 2) -> Dict[str, Dict[str, float]]:
    r, c = tokenize(reference), tokenize(candidate)
    out = {f"rouge-{i}": rouge_n(r, c, i) for i in range(1, n + 1)}
    out["rouge-l"] = rouge_l(r, c)
    return out


def evaluate_pairs(pairs: List[dict]) -> Dict:
    keys = ("rouge-1", "rouge-2", "rouge-l")
    agg = {k: {"precision": 0.0, "recall": 0.0, "f1": 0.0} for k in keys}
    per = []
    for it in pairs:
        s = compute_rouge(it["reference"], it["candidate"])
        per.append({**it, "scores": s})
        for k in keys:
            for m in ("precision", "recall", "f1"):
                agg[k][m] += s[k][m]
    n = max(len(pairs), 1)
    return {"num_samples": len(pairs), "aggregate": {k: {m: v / n for m, v in d.items()} for k, d in agg.items()},
            "per_item": per}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="ROUGE evaluation of reference/candidate pairs")
    p.add_argument("--data_path", type=str, required=True)
    p.add_argument("--output", type=str, default=None)
    a = p.parse_args(argv)
    with open(a.data_path, encoding="utf-8") as fh:
        pairs = [json.loads(x) for x in fh if x.strip()]
    res = evaluate_pairs(pairs)
    for k, v in res["aggregate"].items():
        print(f"{k}: P={v['precision']:.4f} R={v['recall']:.4f} F1={v['f1']:.4f}")
    write_json(a.output, res)


if __name__ == "__main__":
    main()
