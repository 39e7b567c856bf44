"""HumanEval pass@k: generate -> extract -> execute -> score.

    python -m astrai_b200.eval.humaneval --param_path MODEL --data_path HumanEval.jsonl
        [--num_samples 200] [--max_tokens 512] [--temperature 0.8] [--top_p 0.95] [--top_k 50]
        [--batch_size 32] [--test_workers 8] [--test_timeout 3.0] [--problems i ...]
        [--generate_only] [--test_only completions.json] [--output results.json]

Parity: scripts/eval/evaluate_humaneval.py of the reference: the same flags
and stages, the same stop sequences, function-body extraction and
de-duplication of samples, pass@k with the unbiased estimator
``1 - C(n-c, k) / C(n, k)`` of Chen et al. (2021) for k in (1, 10, 100)
whenever k <= n, and a ``_summary`` of the mean pass@k.

Two deliberate differences. (1) Each program run is prompt + completion +
the problem's ``test`` + ``check(entry_point)``: HumanEval's test field only
*defines* ``check``, so a run without the call would pass any completion that
parses. (2) All problems' samples are submitted to the continuous-batching
engine together (:mod:`astrai_b200.eval.generation`).
"""

from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
from concurrent.futures import ProcessPoolExecutor
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from astrai_b200.eval.common import write_json

STOP_SEQUENCES = ("\nclass ", "\ndef ", "\n# ", "\nif __name__", "\nprint(", "\n\n\n")
K_VALUES = (1, 10, 100)


@dataclass
class EvalConfig:
    param_path: str = "./params"
    data_path: str = "./humaneval/HumanEval.jsonl"
    output: Optional[str] = None
    test_only: Optional[str] = None
    generate_only: bool = False
    num_samples: int = 200
    max_tokens: int = 512
    temperature: float = 0.8
    top_p: float = 0.95
    top_k: int = 50
    batch_size: int = 32
    test_timeout: float = 3.0
    test_workers: int = 8
    k_values: Tuple[int, ...] = K_VALUES
    problem_indices: Optional[List[int]] = None


def load_jsonl(path: str) -> List[dict]:
    with open(path, encoding="utf-8") as fh:
        return [json.loads(x) for x in fh if x.strip()]


def trim_stop(text: str) -> str:
    cut = min((i for i in (text.find(s) for s in STOP_SEQUENCES) if i >= 0), default=-1)
    return text if cut < 0 else text[:cut]


def extract_body(code: str, entry_point: str) -> Optional[str]:
    """If the completion re-declares ``entry_point``, keep only that function's indented body."""
    m = re.search(rf"def\s+{re.escape(entry_point)}\b[^:]*:", code)
    if not m:
        return code
    body: List[str] = []
    for line in code[m.end():].split("\n"):
        s = line.rstrip()
        if not s:
            if body:
                body.append("")
            continue
        if body and not s[0].isspace():
            break  # first non-indented line after the body ends it
        if not body and not s[0].isspace():
            break
        body.append(s)
    text = "\n".join(body)
    return text if text.strip() else None


def unique(seq: Sequence[str]) -> List[str]:
    seen = set()
    return [x for x in seq if not (x in seen or seen.add(x))]


def completions_for(raw: Sequence[str], entry_point: str) -> List[str]:
    bodies = [extract_body(trim_stop(r), entry_point) for r in raw]
    return [b for b in bodies if b]


def program(item: dict, completion: str) -> str:
    return f"{item['prompt']}{completion}\n{item['test']}\ncheck({item['entry_point']})\n"


def run_program(args: Tuple[str, float]) -> bool:
    code, timeout = args
    try:
        return subprocess.run([sys.executable, "-c", code], capture_output=True, timeout=timeout).returncode == 0
    except (subprocess.TimeoutExpired, OSError):
        return False


def pass_at_k(n: int, c: int, k: int) -> float:
    if n - c < k:
        return 1.0
    return float(1.0 - np.prod(1.0 - k / np.arange(n - c + 1, n + 1)))


def test_all(items: Sequence[dict], timeout: float, workers: int) -> List[Tuple[str, int, int]]:
    jobs = [(i, (program(it, c), timeout)) for i, it in enumerate(items) for c in it["completions"]]
    passed = [0] * len(items)
    with ProcessPoolExecutor(max_workers=workers) as pool:
        for (i, _), ok in zip(jobs, pool.map(run_program, [j for _, j in jobs])):
            passed[i] += int(ok)
    return [(it["task_id"], len(it["completions"]), p) for it, p in zip(items, passed)]


def score(results: Sequence[Tuple[str, int, int]], k_values=K_VALUES) -> Dict:
    out: Dict[str, dict] = {}
    per_k: Dict[int, List[float]] = {k: [] for k in k_values}
    for tid, n, c in results:
        e = {"task_id": tid, "n": n, "passed": c}
        for k in k_values:
            v = round(pass_at_k(n, c, k), 4) if k <= n else None
            e[f"pass@{k}"] = v
            if v is not None:
                per_k[k].append(v)
        out[tid] = e
    out["_summary"] = {f"pass@{k}": (round(float(np.mean(v)), 4) if v else None) for k, v in per_k.items()}
    return out


def generate(cfg: EvalConfig, problems: Sequence[dict]) -> List[dict]:
    from astrai_b200.eval.generation import create_engine, generate_many

    engine, _ = create_engine(cfg.param_path, cfg.batch_size)
    try:
        prompts = [p["prompt"] for p in problems for _ in range(cfg.num_samples)]
        raw = generate_many(engine, prompts, cfg.max_tokens, cfg.temperature, cfg.top_p, cfg.top_k)
    finally:
        engine.shutdown()
    items = []
    for j, p in enumerate(problems):
        mine = unique(raw[j * cfg.num_samples:(j + 1) * cfg.num_samples])
        items.append({"task_id": p["task_id"], "entry_point": p["entry_point"], "prompt": p["prompt"],
                      "test": p["test"], "completions": completions_for(mine, p["entry_point"])})
    return items


def run(cfg: EvalConfig) -> Dict:
    if cfg.test_only:
        with open(cfg.test_only, encoding="utf-8") as fh:
            items = json.load(fh)
    else:
        problems = load_jsonl(cfg.data_path)
        if cfg.problem_indices:
            problems = [problems[i] for i in cfg.problem_indices]
        items = generate(cfg, problems)
        if cfg.generate_only:
            write_json(cfg.output or "humaneval_completions.json", items)
            return {"completions": len(items)}
    res = score(test_all(items, cfg.test_timeout, cfg.test_workers), cfg.k_values)
    write_json(cfg.output, res)
    for k, v in res["_summary"].items():
        print(f"{k}: {v}")
    return res


def parse_args(argv=None) -> EvalConfig:
    p = argparse.ArgumentParser(description="HumanEval evaluation")
    p.add_argument("--param_path", type=str, default="./params")
    p.add_argument("--data_path", type=str, default="./humaneval/HumanEval.jsonl")
    p.add_argument("--output", type=str, default=None)
    p.add_argument("--test_only", type=str, default=None, help="score a completions JSON written by --generate_only")
    p.add_argument("--generate_only", action="store_true")
    p.add_argument("--num_samples", type=int, default=200)
    p.add_argument("--max_tokens", type=int, default=512)
    p.add_argument("--temperature", type=float, default=0.8)
    p.add_argument("--top_p", type=float, default=0.95)
    p.add_argument("--top_k", type=int, default=50)
    p.add_argument("--batch_size", type=int, default=32)
    p.add_argument("--test_workers", type=int, default=8)
    p.add_argument("--test_timeout", type=float, default=3.0)
    p.add_argument("--problems", type=int, nargs="+", default=None)
    a = p.parse_args(argv)
    return EvalConfig(param_path=a.param_path, data_path=a.data_path, output=a.output, test_only=a.test_only,
                      generate_only=a.generate_only, num_samples=a.num_samples, max_tokens=a.max_tokens,
                      temperature=a.temperature, top_p=a.top_p, top_k=a.top_k, batch_size=a.batch_size,
                      test_timeout=a.test_timeout, test_workers=a.test_workers, problem_indices=a.problems)


def main(argv=None) -> None:
    if not os.environ.get("ASTRAI_ALLOW_CODE_EXECUTION", "1") == "1":
        raise SystemExit("code execution disabled by ASTRAI_ALLOW_CODE_EXECUTION=0")
    run(parse_args(argv))


if __name__ == "__main__":
    main()
