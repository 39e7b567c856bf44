"""MMLU by log-likelihood ranking of the answer letters.

    python -m astrai_b200.eval.mmlu --param_path MODEL --data_dir MMLU_DIR [--n_shot 5] [--split test|val]
        [--subjects ...] [--seed 0] [--output results.json]

Parity: scripts/eval/evaluate_mmlu.py of the reference: the same data layout
(``{data_dir}/{split}/{subject}_{split}.csv`` and ``dev/{subject}_dev.csv``
few-shot rows of question, four options with optional ``A)`` prefixes,
answer letter), the same prompt text and chat-template wrapping of few-shot
exchanges, the same per-subject option shuffling (``random.Random(seed)``
consumed once per question; ``--seed -1`` disables it) and the same results
JSON (per subject accuracy/correct/total and ``_overall``).

Execution differs: when every answer letter is one token, a question costs
one packed forward (the four letters read the same next-token row of
:func:`astrai_b200.eval.loglik.next_token_logprobs`) instead of four, and a
whole subject is scored in packed batches. Subjects are discovered from the
files present (no download: this build runs offline; ``--download`` uses the
``datasets`` package when it is importable).
"""

from __future__ import annotations

import argparse
import csv
import glob
import os
import random
from collections import defaultdict
from typing import Dict, List, Optional, Tuple

from astrai_b200.eval.common import default_device, default_dtype, load_model, write_json
from astrai_b200.eval.loglik import Doc, fit, next_token_logprobs, score_docs

LETTERS = ("A", "B", "C", "D")


def load_csv(path: str) -> List[dict]:
    rows = []
    with open(path, encoding="utf-8") as fh:
        for r in csv.reader(fh):
            if len(r) < 6 or r[0].strip().lower() == "question":
                continue
            item = {"question": r[0].strip(), "answer": r[5].strip()}
            for k, cell in zip(LETTERS, r[1:5]):
                cell = cell.strip()
                item[k] = cell[2:].strip() if cell.startswith(k + ")") else cell
            rows.append(item)
    return rows


def subjects_in(data_dir: str, split: str) -> List[str]:
    suffix = f"_{split}.csv"
    return sorted(os.path.basename(p)[:-len(suffix)] for p in glob.glob(os.path.join(data_dir, split, "*" + suffix)))


def build_prompt(question: str, options: dict, subject: str) -> str:
    lines = [f"The following are multiple choice questions (with answers) about {subject}.", "",
             f"Question: {question}"]
    lines += [f"{k}. {options[k]}" for k in LETTERS]
    return "\n".join(lines) + "\nAnswer:"


def chat_context(tokenizer, prompt: str, subject: str, shots: List[dict]) -> str:
    msgs = []
    for ex in shots:
        msgs.append({"role": "user", "content": build_prompt(ex["question"], ex, subject)})
        msgs.append({"role": "assistant", "content": ex["answer"]})
    msgs.append({"role": "user", "content": prompt})
    return tokenizer.apply_chat_template(msgs, tokenize=False, add_generation_prompt=True)


def shuffle_options(item: dict, rng: random.Random) -> Tuple[dict, str]:
    """Options re-lettered by a random permutation; returns (item, new answer letter)."""
    perm = list(LETTERS)
    rng.shuffle(perm)
    out = {"question": item["question"]}
    for new, old in zip(LETTERS, perm):
        out[new] = item[old]
    return out, LETTERS[perm.index(item["answer"])]


def score_subject(model, tokenizer, subject: str, test: List[dict], dev: Optional[List[dict]], n_shot: int,
                  seed: int = 0, max_len: Optional[int] = None, max_tokens: int = 16384) -> Tuple[float, int, int]:
    max_len = max_len or model.config.max_position_embeddings
    rng = random.Random(seed) if seed >= 0 else None
    shots = (dev or [])[:n_shot] if n_shot > 0 else []
    contexts, answers = [], []
    for item in test:
        it, ans = shuffle_options(item, rng) if rng is not None else (item, item["answer"])
        contexts.append(tokenizer.encode(chat_context(tokenizer, build_prompt(it["question"], it, subject), subject,
                                                      shots)))
        answers.append(ans)
    letter_ids = [tokenizer.encode(k, add_special_tokens=False) for k in LETTERS]
    if all(len(t) == 1 for t in letter_ids):
        lsm = next_token_logprobs(model, contexts, max_len=max_len, max_tokens=max_tokens)
        scores = lsm[:, [t[0] for t in letter_ids]]  # [Q, 4]
    else:
        docs = [fit(c, t, max_len) for c in contexts for t in letter_ids]
        lp = score_docs(model, docs, max_len=max_len, max_tokens=max_tokens)
        import torch

        scores = torch.tensor([float(x.sum()) for x in lp]).view(len(contexts), 4)
    pred = scores.argmax(-1).tolist()
    correct = sum(1 for p, a in zip(pred, answers) if LETTERS[p] == a)
    return (correct / len(test) if test else 0.0), correct, len(test)


def download(data_dir: str) -> None:
    try:
        from datasets import load_dataset
    except ImportError as e:
        raise RuntimeError("MMLU download needs the `datasets` package and network access; place the CSV files "
                           f"under {data_dir}/{{dev,val,test}}/ instead") from e
    for local, hf in (("dev", "dev"), ("val", "validation"), ("test", "test")):
        grouped: Dict[str, list] = defaultdict(list)
        for it in load_dataset("cais/mmlu", "all", split=hf):
            ch = it["choices"]
            grouped[it["subject"]].append([it["question"], *(f"{k}){c}" for k, c in zip(LETTERS, ch)),
                                           LETTERS[it["answer"]]])
        os.makedirs(os.path.join(data_dir, local), exist_ok=True)
        for subject, rows in grouped.items():
            with open(os.path.join(data_dir, local, f"{subject}_{local}.csv"), "w", encoding="utf-8",
                      newline="") as fh:
                csv.writer(fh).writerows(rows)


def run(model, tokenizer, data_dir: str, split: str = "test", n_shot: int = 5, subjects=None, seed: int = 0,
        output: Optional[str] = None) -> Dict:
    results: Dict[str, dict] = {}
    tot_c = tot_n = 0
    for subject in subjects or subjects_in(data_dir, split):
        test_path = os.path.join(data_dir, split, f"{subject}_{split}.csv")
        if not os.path.exists(test_path):
            print(f"  skipping {subject}: {test_path} not found")
            continue
        dev_path = os.path.join(data_dir, "dev", f"{subject}_dev.csv")
        dev = load_csv(dev_path) if os.path.exists(dev_path) else None
        acc, c, n = score_subject(model, tokenizer, subject, load_csv(test_path), dev, n_shot, seed)
        results[subject] = {"accuracy": round(acc, 4), "correct": c, "total": n}
        tot_c, tot_n = tot_c + c, tot_n + n
        print(f"  {subject:40s} {acc:7.2%} ({c}/{n})")
    overall = tot_c / tot_n if tot_n else 0.0
    results["_overall"] = {"accuracy": round(overall, 4), "correct": tot_c, "total": tot_n}
    print(f"  overall {overall:.2%} ({tot_c}/{tot_n})")
    write_json(output, results)
    return results


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="MMLU evaluation")
    p.add_argument("--param_path", type=str, default="./params")
    p.add_argument("--data_dir", type=str, default="./mmlu_data")
    p.add_argument("--download", action="store_true")
    p.add_argument("--n_shot", type=int, default=5)
    p.add_argument("--subjects", type=str, nargs="+")
    p.add_argument("--output", type=str)
    p.add_argument("--split", type=str, default="test", choices=["test", "val"])
    p.add_argument("--device", type=str, default=default_device())
    p.add_argument("--dtype", type=str, default=default_dtype())
    p.add_argument("--seed", type=int, default=0, help="option shuffling seed (-1 disables)")
    a = p.parse_args(argv)
    if a.download or not os.path.exists(a.data_dir):
        download(a.data_dir)
    model, tok = load_model(a.param_path, a.device, a.dtype)
    run(model, tok, a.data_dir, a.split, a.n_shot, a.subjects, a.seed, a.output)


if __name__ == "__main__":
    main()
