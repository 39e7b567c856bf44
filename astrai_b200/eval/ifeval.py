"""IFEval: verifiable instruction following (Zhou et al., 2023).

    python -m astrai_b200.eval.ifeval --param_path MODEL --data_path input_data.jsonl [--output results.json]
        [--max_tokens 512] [--temperature 0.1] [--top_p 0.95] [--top_k 50] [--num_samples 1]
        [--batch_size 1] [--limit N] [--dump_responses responses.jsonl]

Each problem has a prompt and a list of ``instruction_id_list`` entries with
``kwargs``; a verifier per instruction id decides whether a response complies.
With several samples a constraint counts as passed if any sample passes.
Parity: scripts/eval/evaluate_ifeval.py of the reference: the same flags,
chat-template prompting, supported ids (every IFEval id except
``language:response_language``, which needs a language detector, plus the
reference's extra ``general_punctuation``, ``number_highlighted_words``,
``start_checker`` and ``nth_word_checker``) and the same results layout
(per-problem constraint rows and a ``_summary`` with per-type accuracy).
Verifiers are written from the benchmark's definitions; ``relation`` kwargs
are "less than" or "at least". All problems are generated as one batched
submission to the engine.
"""

from __future__ import annotations

import argparse
import json
import re
from typing import Callable, Dict, List, Optional

from astrai_b200.eval.common import write_json

VERIFIERS: Dict[str, Callable[[str, dict], bool]] = {}


def verifier(instruction_id: str):
    def deco(fn):
        VERIFIERS[instruction_id] = fn
        return fn

    return deco


def _compare(count: int, target: int, relation: Optional[str]) -> bool:
    return count < target if relation == "less than" else count >= target


def _words(text: str) -> List[str]:
    return re.findall(r"\b\w+\b", text)


def _sentences(text: str) -> List[str]:
    return [s for s in re.split(r"(?<=[.!?])\s+", text.strip()) if s.strip()] if text.strip() else []


@verifier("keywords:existence")
def _kw_exist(r, kw):
    return all(re.search(re.escape(k), r, re.I) for k in kw["keywords"])


@verifier("keywords:frequency")
def _kw_freq(r, kw):
    return _compare(len(re.findall(re.escape(kw["keyword"]), r, re.I)), kw.get("frequency", 1), kw.get("relation"))


@verifier("keywords:forbidden_words")
def _kw_forbid(r, kw):
    return not any(re.search(rf"\b{re.escape(w)}\b", r, re.I) for w in kw["forbidden_words"])


@verifier("keywords:letter_frequency")
def _letter_freq(r, kw):
    return _compare(r.lower().count(kw["letter"].lower()), kw.get("let_frequency", 1), kw.get("let_relation"))


@verifier("detectable_content:number_placeholders")
def _placeholders(r, kw):
    return len(re.findall(r"\[[^\]]*\]", r)) >= kw.get("num_placeholders", 1)


@verifier("detectable_content:postscript")
def _postscript(r, kw):
    marker = kw.get("postscript_marker", "P.S.").strip()
    if marker.upper().rstrip(".") == "P.P.S":
        pat = r"p\.\s?p\.\s?s"
    elif marker.upper().rstrip(".") == "P.S":
        pat = r"p\.\s?s\."
    else:
        pat = re.escape(marker.lower())
    return re.search(pat, r.lower()) is not None


@verifier("detectable_format:number_bullet_lists")
def _bullets(r, kw):
    stars = re.findall(r"^\s*\*[^*].*$", r, re.M)
    dashes = re.findall(r"^\s*-.*$", r, re.M)
    return len(stars) + len(dashes) == kw.get("num_bullets", 1)


@verifier("detectable_format:number_highlighted_sections")
def _highlights(r, kw):
    return sum(1 for h in re.findall(r"\*[^\n*]+\*", r) if h.strip("*").strip()) >= kw.get("num_highlights", 1)


@verifier("detectable_format:multiple_sections")
def _sections(r, kw):
    parts = re.split(r"\s?" + re.escape(kw.get("section_spliter", "Section")) + r"\s?\d+\s?", r)
    return len(parts) - 1 >= kw.get("num_sections", 1)


@verifier("detectable_format:title")
def _title(r, kw):
    return any(t.strip("<>").strip() for t in re.findall(r"<<[^>\n]+>>", r))


@verifier("detectable_format:json_format")
def _json(r, kw):
    v = r.strip()
    v = re.sub(r"^```(?:json)?", "", v, flags=re.I).strip()
    v = v[:-3].strip() if v.endswith("```") else v
    try:
        json.loads(v)
        return True
    except ValueError:
        return False


@verifier("detectable_format:constrained_response")
def _constrained(r, kw):
    return any(opt in r for opt in ("My answer is yes.", "My answer is no.", "My answer is maybe."))


@verifier("detectable_format:general_punctuation")
def _punct(r, kw):
    return not any(p in r for p in kw.get("punctuation_blacklist", []))


@verifier("detectable_format:number_highlighted_words")
def _hl_words(r, kw):
    return len(re.findall(r"\*[^\s*][^*]*[^\s*]\*", r)) >= kw.get("num_highlights", 1)


@verifier("startend:end_checker")
def _end(r, kw):
    return r.strip().rstrip('"').rstrip().lower().endswith(kw["end_phrase"].strip().lower())


@verifier("startend:quotation")
def _quoted(r, kw):
    v = r.strip()
    return len(v) >= 2 and v[0] == '"' and v[-1] == '"'


@verifier("startend:start_checker")
def _start(r, kw):
    return re.search(r"^\s*" + re.escape(kw["starter"]), r, re.M) is not None


@verifier("change_case:english_capital")
def _upper(r, kw):
    return r.isupper()


@verifier("change_case:english_lowercase")
def _lower(r, kw):
    return r.islower()


@verifier("change_case:capital_word_frequency")
def _caps(r, kw):
    return _compare(len(re.findall(r"\b[A-Z]{2,}\b", r)), kw.get("capital_frequency", 1), kw.get("capital_relation"))


@verifier("punctuation:no_comma")
def _no_comma(r, kw):
    return "," not in r


@verifier("length_constraints:number_words")
def _n_words(r, kw):
    return _compare(len(_words(r)), kw.get("num_words", 100), kw.get("relation"))


@verifier("length_constraints:number_sentences")
def _n_sent(r, kw):
    return _compare(len(_sentences(r)), kw.get("num_sentences", 5), kw.get("relation"))


def _paragraphs(r: str) -> List[str]:
    parts = re.split(r"\s?\*\*\*\s?", r) if "***" in r else re.split(r"\n\n+", r)
    return [p.strip() for p in parts if p.strip()]


@verifier("length_constraints:number_paragraphs")
def _n_para(r, kw):
    return len(_paragraphs(r)) == kw.get("num_paragraphs", 1)


@verifier("length_constraints:nth_paragraph_first_word")
def _nth_para(r, kw):
    paras = [p.strip() for p in re.split(r"\n\n+", r) if p.strip()]
    n, nth = kw.get("num_paragraphs", 1), kw.get("nth_paragraph", 1)
    if len(paras) != n or nth > n or not paras[nth - 1].split():
        return False
    first = paras[nth - 1].split()[0].strip().lstrip("'\"").rstrip(".,!?:;\"'")
    return first.lower() == kw.get("first_word", "").lower()


@verifier("length_constraints:nth_word_checker")
def _nth_word(r, kw):
    w = _words(r)
    n = kw.get("nth_word", 1)
    return n <= len(w) and w[n - 1].lower() == kw.get("target_word", "").lower()


@verifier("combination:repeat_prompt")
def _repeat(r, kw):
    return r.strip().lower().startswith(kw["prompt_to_repeat"].strip().lower())


@verifier("combination:two_responses")
def _two(r, kw):
    parts = [p.strip() for p in r.split("******") if p.strip()]
    return len(parts) == 2 and parts[0] != parts[1]


def verify(response: str, instruction_id: str, kwargs: dict) -> Optional[bool]:
    """True / False, or None when the id has no verifier; a verifier error counts as False."""
    fn = VERIFIERS.get(instruction_id)
    if fn is None:
        return None
    try:
        return bool(fn(response, {k: v for k, v in (kwargs or {}).items() if v is not None}))
    except (KeyError, TypeError, ValueError, re.error):
        return False


def score(problems: List[dict], responses: List[List[str]]) -> Dict:
    """``responses[i]`` = samples for ``problems[i]``."""
    results: Dict[str, dict] = {}
    per_type: Dict[str, List[int]] = {}
    tot_v = tot_p = unsupported = 0
    for prob, samples in zip(problems, responses):
        rows, passed, verified = [], 0, 0
        kw_list = prob.get("kwargs", [])
        for j, iid in enumerate(prob["instruction_id_list"]):
            kw = kw_list[j] if j < len(kw_list) else {}
            ok = any(verify(s, iid, kw) for s in samples)
            sup = iid in VERIFIERS
            if sup:
                verified += 1
                passed += int(ok)
                t = per_type.setdefault(iid, [0, 0])
                t[0] += 1
                t[1] += int(ok)
            else:
                unsupported += 1
            rows.append({"instruction_id": iid, "passed": ok, "supported": sup, "kwargs": kw})
        tot_v += verified
        tot_p += passed
        results[str(prob["key"])] = {
            "key": prob["key"], "prompt": prob["prompt"], "response": samples[0] if samples else "",
            "num_samples": len(samples), "num_constraints": len(rows), "num_verified": verified,
            "num_passed": passed, "accuracy": round(passed / verified, 4) if verified else None, "constraints": rows}
    results["_summary"] = {
        "total_problems": len(problems), "total_constraints": tot_v, "total_passed": tot_p,
        "overall_accuracy": round(tot_p / tot_v, 4) if tot_v else 0.0, "unsupported_constraints": unsupported,
        "supported_types": sorted(VERIFIERS),
        "per_type_accuracy": {k: {"total": n, "passed": p, "accuracy": round(p / n, 4) if n else 0.0}
                              for k, (n, p) in sorted(per_type.items())}}
    return results


def evaluate(engine, tokenizer, problems: List[dict], max_tokens: int = 512, temperature: float = 0.1,
             top_p: float = 0.95, top_k: int = 50, num_samples: int = 1) -> Dict:
    from astrai_b200.eval.generation import generate_many

    prompts = [tokenizer.apply_chat_template([{"role": "user", "content": p["prompt"]}], tokenize=False,
                                             add_generation_prompt=True) for p in problems]
    flat = generate_many(engine, [x for x in prompts for _ in range(num_samples)], max_tokens, temperature, top_p,
                         top_k)
    return score(problems, [flat[i * num_samples:(i + 1) * num_samples] for i in range(len(problems))])


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="IFEval evaluation")
    p.add_argument("--param_path", type=str, default="./params")
    p.add_argument("--data_path", type=str, default="./ifeval/input_data.jsonl")
    p.add_argument("--output", type=str, default=None)
    p.add_argument("--max_tokens", type=int, default=512)
    p.add_argument("--temperature", type=float, default=0.1)
    p.add_argument("--top_p", type=float, default=0.95)
    p.add_argument("--top_k", type=int, default=50)
    p.add_argument("--num_samples", type=int, default=1)
    p.add_argument("--batch_size", type=int, default=1)
    p.add_argument("--limit", type=int, default=None)
    p.add_argument("--dump_responses", type=str, default=None)
    a = p.parse_args(argv)
    from astrai_b200.eval.common import load_items
    from astrai_b200.eval.generation import create_engine

    problems = load_items(a.data_path)[:a.limit] if a.limit else load_items(a.data_path)
    engine, tok = create_engine(a.param_path, a.batch_size)
    try:
        res = evaluate(engine, tok, problems, a.max_tokens, a.temperature, a.top_p, a.top_k, a.num_samples)
    finally:
        engine.shutdown()
    if a.dump_responses:
        with open(a.dump_responses, "w", encoding="utf-8") as fh:
            for k, v in res.items():
                if not k.startswith("_"):
                    fh.write(json.dumps({"key": v["key"], "prompt": v["prompt"], "response": v["response"]},
                                        ensure_ascii=False) + "\n")
    s = res["_summary"]
    print(f"problems={s['total_problems']} constraints={s['total_constraints']} accuracy={s['overall_accuracy']}")
    write_json(a.output, res)


if __name__ == "__main__":
    main()
