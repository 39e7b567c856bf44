"""IFD (instruction-following difficulty) scoring of instruction/response data.

    python -m astrai_b200.eval.ifd --param_path MODEL --input_path DATA --output_dir OUT
        [--format plain|messages] [--instr_key instruction] [--resp_key response] [--max_len 2048]
        [--batch_size 8] [--sentinel_text "\\n"] [--per_token] [--max_samples N]

IFD = mean NLL of the response given the instruction / mean NLL of the same
response tokens given only a short sentinel prefix (default ``"\\n"``; empty
falls back to the bos / pad / eos token). Parity: scripts/eval/evaluate_ifd.py
of the reference: the same flags, truncation rule (response capped at half of
``max_len``, context cut from the left), ``messages`` format (one score per
assistant turn, context = earlier turns joined by blank lines, sample score =
mean over turns), per-file ``{label}_ifd.jsonl`` rows with ``ifd`` and
``ifd_detail`` (L_cond, L_uncond, ifd, ctx_len, resp_len, optional
ifd_per_token) and a ``summary.json`` (samples, valid_ifd, skipped,
mean/median/stdev/min/max).

Execution: conditional and unconditional documents of a whole batch go
through one packed scorer (:mod:`astrai_b200.eval.loglik`): segment ids keep
packed documents apart, so neither pass builds a dense mask or pads.
"""

from __future__ import annotations

import argparse
import json
import os
import random
import statistics
from typing import Dict, List, Optional, Sequence, Tuple

from astrai_b200.eval.common import collect_input_files, default_device, default_dtype, load_items, load_model, write_json
from astrai_b200.eval.loglik import Doc, score_docs


def sentinel_ids(tokenizer, text: str) -> List[int]:
    if text:
        ids = tokenizer.encode(text, add_special_tokens=False)
        if ids:
            return ids
    for name in ("bos_token_id", "pad_token_id", "eos_token_id"):
        tid = getattr(tokenizer, name, None)
        if tid is not None:
            return [tid]
    return [0]


def trim(ctx: List[int], resp: List[int], max_len: int) -> Tuple[List[int], List[int]]:
    resp = resp[:max_len // 2] if len(resp) > max_len // 2 else resp
    over = len(ctx) + len(resp) - max_len
    if over <= 0:
        return ctx, resp
    if over >= len(ctx):
        return [], resp[:max_len]
    return ctx[over:], resp


def score_pairs(model, pairs: Sequence[Tuple[List[int], List[int]]], sentinel: List[int], max_len: int = 2048,
                max_tokens: int = 16384, per_token: bool = False) -> List[Optional[dict]]:
    """IFD detail for each (context ids, response ids) pair; None when either side is empty."""
    live = [i for i, (c, r) in enumerate(pairs) if c and r]
    docs = [Doc(list(pairs[i][0]) + list(pairs[i][1]), len(pairs[i][0])) for i in live]
    docs += [Doc(list(sentinel) + list(pairs[i][1]), len(sentinel)) for i in live]
    lps = score_docs(model, docs, max_len=max_len + len(sentinel), max_tokens=max_tokens)
    out: List[Optional[dict]] = [None] * len(pairs)
    n = len(live)
    for k, i in enumerate(live):
        cond, unc = -lps[k], -lps[n + k]
        lc, lu = float(cond.mean()), float(unc.mean())
        d = {"L_cond": round(lc, 6), "L_uncond": round(lu, 6), "ifd": round(lc / lu, 6) if lu > 0 else None,
             "ctx_len": len(pairs[i][0]), "resp_len": len(pairs[i][1])}
        if per_token:
            d["ifd_per_token"] = [round(float(c) / float(u), 6) if float(u) > 0 else None for c, u in zip(cond, unc)]
        out[i] = d
    return out


def _turns(item: dict, tokenizer, fmt: str, instr_key: str, resp_key: str, max_len: int):
    if fmt == "messages":
        msgs = item.get("messages", [])
        turns = []
        for i, m in enumerate(msgs):
            if m.get("role") != "assistant":
                continue
            ctx = tokenizer.encode("\n\n".join(x["content"] for x in msgs[:i]))
            resp = tokenizer.encode(m["content"], add_special_tokens=False)
            c, r = trim(ctx, resp, max_len)
            if c and r:
                turns.append((c, r))
        return turns
    c, r = trim(tokenizer.encode(item[instr_key], add_special_tokens=False),
                tokenizer.encode(item[resp_key], add_special_tokens=False), max_len)
    return [(c, r)] if c and r else []


def score_items(model, tokenizer, items: List[dict], fmt: str = "plain", instr_key: str = "instruction",
                resp_key: str = "response", max_len: int = 2048, batch_size: int = 8, sentinel_text: str = "\n",
                per_token: bool = False) -> List[dict]:
    sent = sentinel_ids(tokenizer, sentinel_text)
    rows: List[dict] = []
    for b in range(0, len(items), batch_size):
        chunk = items[b:b + batch_size]
        turns = [_turns(it, tokenizer, fmt, instr_key, resp_key, max_len) for it in chunk]
        flat = [t for ts in turns for t in ts]
        scores = score_pairs(model, flat, sent, max_len, max_tokens=batch_size * max_len, per_token=per_token)
        at = 0
        for it, ts in zip(chunk, turns):
            sc = scores[at:at + len(ts)]
            at += len(ts)
            if fmt == "messages":
                if not ts:
                    rows.append({**it, "ifd": None, "skip_reason": "no valid assistant turns", "ifd_turns": []})
                    continue
                valid = [s for s in sc if s is not None and s.get("ifd") is not None]
                avg = sum(s["ifd"] for s in valid) / len(valid) if valid else None
                rows.append({**it, "ifd": avg, "ifd_detail": valid[0] if len(valid) == 1 else None, "ifd_turns": sc})
            elif not ts:
                rows.append({**it, "ifd": None, "ifd_detail": {"skip_reason": "empty ctx or resp"}})
            else:
                rows.append({**it, "ifd": sc[0]["ifd"], "ifd_detail": sc[0]})
    return rows


def summarize(rows: List[dict]) -> Dict:
    vals = [r["ifd"] for r in rows if r.get("ifd") is not None]
    st = {"samples": len(rows), "valid_ifd": len(vals), "skipped": len(rows) - len(vals)}
    if vals:
        st.update(mean_ifd=statistics.mean(vals), median_ifd=statistics.median(vals), min_ifd=min(vals),
                  max_ifd=max(vals))
        if len(vals) > 1:
            st["stdev_ifd"] = statistics.stdev(vals)
    return st


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="Compute IFD scores for instruction-response data")
    p.add_argument("--param_path", type=str, required=True)
    p.add_argument("--input_path", type=str, required=True)
    p.add_argument("--output_dir", type=str, required=True)
    p.add_argument("--max_len", type=int, default=2048)
    p.add_argument("--format", type=str, default="plain", choices=["plain", "messages"])
    p.add_argument("--instr_key", type=str, default="instruction")
    p.add_argument("--resp_key", type=str, default="response")
    p.add_argument("--batch_size", type=int, default=8)
    p.add_argument("--device", type=str, default=None)
    p.add_argument("--dtype", type=str, default=default_dtype())
    p.add_argument("--sentinel_text", type=str, default="\n")
    p.add_argument("--per_token", action="store_true")
    p.add_argument("--max_samples", type=int, default=None)
    a = p.parse_args(argv)
    model, tok = load_model(a.param_path, a.device or default_device(), a.dtype)
    os.makedirs(a.output_dir, exist_ok=True)
    summary = {}
    for path in collect_input_files(a.input_path):
        label = os.path.splitext(os.path.basename(path))[0]
        items = load_items(path)
        if a.max_samples and len(items) > a.max_samples:
            items = random.sample(items, a.max_samples)
        rows = score_items(model, tok, items, a.format, a.instr_key, a.resp_key, a.max_len, a.batch_size,
                           a.sentinel_text, a.per_token)
        with open(os.path.join(a.output_dir, f"{label}_ifd.jsonl"), "w", encoding="utf-8") as fh:
            for r in rows:
                fh.write(json.dumps(r, ensure_ascii=False) + "\n")
        summary[label] = summarize(rows)
        print(f"[{label}] {summary[label]}")
    write_json(os.path.join(a.output_dir, "summary.json"), summary)


if __name__ == "__main__":
    main()
