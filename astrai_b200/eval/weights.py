"""SVD effective-rank and weight statistics of a checkpoint.

    python -m astrai_b200.eval.weights --ckpt_dir CKPT [--compare CKPT2 ...] [--no_svd] [--output stats.json]

Parity: scripts/eval/analyze_weights.py of the reference: per ``*.weight``
tensor of ``model.safetensors`` the metrics er_90/er_95/er_99 (smallest rank
holding that share of the squared singular values) and their ratios to
min(shape), the entropic rank exp(H(sigma^2 / sum sigma^2)), top-1 / top-5
singular-value shares, decay ratio and condition number, plus mean / std /
min / max; a per-component summary (layers.*.<module>.<param> grouped by
module) and a JSON dump.

Execution: tensors of equal shape are stacked and their singular values
computed as one batched ``torch.linalg.svdvals`` in fp32 on the GPU when one
is present (24 layers of q_proj are one call, not 24).
"""

from __future__ import annotations

import argparse
import json
import math
import os
from collections import defaultdict
from typing import Dict, List

import torch

from astrai_b200.eval.common import write_json


def spectrum_metrics(s: torch.Tensor, shape) -> dict:
    """Metrics from singular values ``s`` (descending) of a matrix of ``shape``."""
    s = s.double()
    e = s * s
    tot = float(e.sum())
    cum = torch.cumsum(e, 0) / tot if tot > 0 else torch.ones_like(e)
    k = min(shape)
    p = e / tot if tot > 0 else e
    p = p[p > 1e-30]
    ent = float(torch.exp(-(p * p.log()).sum())) if p.numel() else 0.0
    ssum = float(s.sum()) or 1.0
    er = {q: int((cum < q / 100).sum()) + 1 for q in (90, 95, 99)}
    return {"shape": tuple(shape), "min_dim": k, "er_90": er[90], "er_95": er[95], "er_99": er[99],
            "er_99_norm": er[99] / k, "er_95_norm": er[95] / k, "entropic_rank": ent, "entropic_rank_norm": ent / k,
            "top1_ratio": float(s[0]) / ssum, "top5_ratio": float(s[:5].sum()) / ssum,
            "decay_ratio": float(s[-1] / s[0]) if s[0] > 0 else 0.0,
            "condition_number": float(s[0] / s[-1]) if s[-1] > 0 else math.inf}


def basic_stats(t: torch.Tensor) -> dict:
    f = t.float()
    return {"mean": float(f.mean()), "std": float(f.std()) if f.numel() > 1 else 0.0, "min": float(f.min()),
            "max": float(f.max())}


def analyze(state: Dict[str, torch.Tensor], svd: bool = True, device=None) -> Dict[str, dict]:
    dev = device or ("cuda" if torch.cuda.is_available() else "cpu")
    keys = sorted(k for k in state if ".weight" in k and "freqs_cis" not in k and "rotary" not in k)
    out = {k: {"shape": tuple(state[k].shape), "is_1d": state[k].ndim == 1, **basic_stats(state[k])} for k in keys}
    if not svd:
        return out
    by_shape: Dict[tuple, List[str]] = defaultdict(list)
    for k in keys:
        if state[k].ndim == 2:
            by_shape[tuple(state[k].shape)].append(k)
    for shape, names in by_shape.items():
        step = max(1, (1 << 28) // (shape[0] * shape[1] * 4))  # <= 1 GiB of fp32 per batched call
        for i in range(0, len(names), step):
            grp = names[i:i + step]
            sv = torch.linalg.svdvals(torch.stack([state[n].to(dev, torch.float32) for n in grp])).cpu()
            for n, s in zip(grp, sv):
                out[n].update(spectrum_metrics(s, shape))
    return out


def component(key: str) -> str:
    parts = key.split(".")
    if parts[0] == "layers" and len(parts) >= 4:
        return ".".join(parts[2:-1]) or parts[2]
    return key


def summarize(results: Dict[str, dict]) -> Dict[str, dict]:
    groups: Dict[str, List[dict]] = defaultdict(list)
    for k, r in results.items():
        if "er_99_norm" in r:
            groups[component(k)].append(r)
    return {c: {"n": len(v), "er_99_norm": sum(r["er_99_norm"] for r in v) / len(v),
                "entropic_rank_norm": sum(r["entropic_rank_norm"] for r in v) / len(v),
                "top1_ratio": sum(r["top1_ratio"] for r in v) / len(v),
                "condition_number": sum(r["condition_number"] for r in v) / len(v)} for c, v in sorted(groups.items())}


def analyze_dir(ckpt_dir: str, svd: bool = True) -> Dict:
    from safetensors.torch import load_file

    path = os.path.join(ckpt_dir, "model.safetensors")
    if not os.path.exists(path):
        raise FileNotFoundError(path)
    meta = {}
    if os.path.exists(os.path.join(ckpt_dir, "meta.json")):
        with open(os.path.join(ckpt_dir, "meta.json")) as fh:
            meta = json.load(fh)
    res = analyze(load_file(path), svd)
    return {"meta": meta, "tensors": res, "components": summarize(res) if svd else {}}


def main(argv=None) -> None:
    p = argparse.ArgumentParser(description="SVD effective rank & weight statistics of a model checkpoint.")
    p.add_argument("--ckpt_dir", type=str, required=True)
    p.add_argument("--compare", type=str, nargs="*")
    p.add_argument("--no_svd", action="store_true")
    p.add_argument("--output", type=str, default=None)
    a = p.parse_args(argv)
    allres = {}
    for label, d in [("base", a.ckpt_dir)] + [(f"compare_{i}", c) for i, c in enumerate(a.compare or [])]:
        r = analyze_dir(d, not a.no_svd)
        allres[label] = {"path": d, **r}
        print(f"== {label}: {d}")
        for c, s in r["components"].items():
            print(f"  {c:28s} n={s['n']:3d} ER@99={s['er_99_norm']:.4f} EntRank={s['entropic_rank_norm']:.4f} "
                  f"top1={s['top1_ratio']:.4f} cond={s['condition_number']:.1f}")
    write_json(a.output, allres)


if __name__ == "__main__":
    main()
