"""Packed log-likelihood scoring: the engine behind the PPL, MMLU and IFD evals.

The reference's scripts run one padded forward per batch of texts
(scripts/eval/evaluate_ppl.py:39-76), one forward per MMLU answer letter
(evaluate_mmlu.py:182-206), and a dense ``[S, S]`` document mask for packed
IFD rows (evaluate_ifd.py:110-137). Here every request is a *document*
``ids`` whose tokens from ``n_ctx`` on are scored. Documents are packed
best-fit-decreasing into rows of ``max_len`` tokens. Inside a row each document
gets its own segment id (the attention kernel keeps a query to keys of its own
segment) and positions that restart at 0. The lm_head runs only at the
positions whose next token is scored, and the log-probabilities come from the
fused logprob kernel, so no ``[tokens, vocab]`` fp32 tensor and no dense mask
is ever built.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, List, Optional, Sequence, Tuple

import torch

from astrai_b200.ops.loss import token_logprobs
from astrai_b200.preprocessing.pipeline import plan_bfd

ROW_ALIGN = 16


@dataclass
class Doc:
    """Token ids; tokens ``ids[n_ctx:]`` are scored (each given everything before it)."""

    ids: List[int]
    n_ctx: int

    def __post_init__(self):
        if self.n_ctx < 1:
            raise ValueError("a scored document needs at least one context token")


def fit(context: Sequence[int], target: Sequence[int], max_len: int) -> Doc:
    """Truncate to ``max_len`` tokens: the target keeps at most ``max_len - 1`` tokens (its head), the
    context is cut from the left; an empty context is invalid (nothing predicts the first target)."""
    target = list(target)[:max_len - 1]
    keep = max_len - len(target)
    context = list(context)[-keep:] if keep > 0 else []
    return Doc(context + target, len(context))


def _rows(docs: Sequence[Doc], max_len: int) -> List[List[int]]:
    return plan_bfd([range(len(d.ids)) for d in docs], max_len)


def _batches(bins: List[List[int]], docs: Sequence[Doc], max_tokens: int) -> Iterable[List[List[int]]]:
    """Group packed rows so that rows x padded row length stays under ``max_tokens``."""
    order = sorted(bins, key=lambda b: -sum(len(docs[i].ids) for i in b))
    cur: List[List[int]] = []
    width = 0
    for b in order:
        n = sum(len(docs[i].ids) for i in b)
        w = max(width, -(-n // ROW_ALIGN) * ROW_ALIGN)
        if cur and w * (len(cur) + 1) > max_tokens:
            yield cur
            cur, w = [], -(-n // ROW_ALIGN) * ROW_ALIGN
        cur.append(b)
        width = w
    if cur:
        yield cur


@torch.inference_mode()
def score_docs(model, docs: Sequence[Doc], max_len: int = 2048, max_tokens: int = 16384,
               device: Optional[torch.device] = None) -> List[torch.Tensor]:
    """Per-token log p for the scored tokens of each document (fp32 CPU tensors, input order)."""
    if not docs:
        return []
    dev = device or next(model.parameters()).device
    for d in docs:
        if len(d.ids) > max_len:
            raise ValueError(f"document of {len(d.ids)} tokens exceeds max_len={max_len}; use fit()")
    out: List[Optional[torch.Tensor]] = [None] * len(docs)
    for rows in _batches(_rows(docs, max_len), docs, max(max_tokens, max_len)):
        width = max(-(-sum(len(docs[i].ids) for i in r) // ROW_ALIGN) * ROW_ALIGN for r in rows)
        B = len(rows)
        ids = torch.zeros(B, width, dtype=torch.long)
        pos = torch.zeros(B, width, dtype=torch.long)
        # padding tokens get unique negative segments: they see only themselves
        seg = -(torch.arange(width, dtype=torch.int32) + 1).repeat(B, 1)
        keep = torch.zeros(B, width, dtype=torch.bool)
        tgt = torch.zeros(B, width, dtype=torch.long)
        spans: List[Tuple[int, int]] = []  # (doc index, n scored) in row-major order of ``keep``
        for r, row in enumerate(rows):
            at = 0
            for j, i in enumerate(sorted(row)):
                d = docs[i]
                n = len(d.ids)
                ids[r, at:at + n] = torch.tensor(d.ids)
                pos[r, at:at + n] = torch.arange(n)
                seg[r, at:at + n] = j
                # position p predicts token p + 1: scored tokens n_ctx..n-1 come from n_ctx-1..n-2
                keep[r, at + d.n_ctx - 1:at + n - 1] = True
                tgt[r, at + d.n_ctx - 1:at + n - 1] = torch.tensor(d.ids[d.n_ctx:])
                at += n
            for i in sorted(row):
                spans.append((i, len(docs[i].ids) - docs[i].n_ctx))
        # the row-major order of ``keep`` visits documents of a row in the order they were laid out
        logits = model(ids.to(dev, non_blocking=True), position_ids=pos.to(dev, non_blocking=True),
                       seg_ids=seg.to(dev, non_blocking=True), logits_to_keep=keep.to(dev))["logits"]
        lp = token_logprobs(logits, tgt[keep].to(dev)).float().cpu()
        at = 0
        for i, n in spans:
            out[i] = lp[at:at + n]
            at += n
    return out  # type: ignore[return-value]


@torch.inference_mode()
def next_token_logprobs(model, contexts: Sequence[Sequence[int]], max_len: int = 2048, max_tokens: int = 16384,
                        device: Optional[torch.device] = None) -> torch.Tensor:
    """log-softmax over the vocabulary of the token following each context: ``[len(contexts), V]`` fp32.

    Multiple-choice scoring with one-token answers needs one forward per question, not one per
    choice: every choice reads the same row.
    """
    dev = device or next(model.parameters()).device
    docs = [Doc(list(c)[-max_len:], 1) for c in contexts]
    rows_out: List[Optional[torch.Tensor]] = [None] * len(docs)
    for rows in _batches(_rows(docs, max_len), docs, max(max_tokens, max_len)):
        width = max(-(-sum(len(docs[i].ids) for i in r) // ROW_ALIGN) * ROW_ALIGN for r in rows)
        B = len(rows)
        ids = torch.zeros(B, width, dtype=torch.long)
        pos = torch.zeros(B, width, dtype=torch.long)
        seg = -(torch.arange(width, dtype=torch.int32) + 1).repeat(B, 1)
        keep = torch.zeros(B, width, dtype=torch.bool)
        order: List[int] = []
        for r, row in enumerate(rows):
            at = 0
            for j, i in enumerate(sorted(row)):
                n = len(docs[i].ids)
                ids[r, at:at + n] = torch.tensor(docs[i].ids)
                pos[r, at:at + n] = torch.arange(n)
                seg[r, at:at + n] = j
                keep[r, at + n - 1] = True
                at += n
                order.append(i)
        logits = model(ids.to(dev), position_ids=pos.to(dev), seg_ids=seg.to(dev),
                       logits_to_keep=keep.to(dev))["logits"]
        lsm = torch.log_softmax(logits.float(), dim=-1).cpu()
        for k, i in enumerate(order):
            rows_out[i] = lsm[k]
    return torch.stack(rows_out)  # type: ignore[arg-type]
