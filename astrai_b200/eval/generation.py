"""Batched generation for the generation-based evals (HumanEval, IFEval).

The reference's scripts call ``engine.generate`` one prompt (or one prompt's
sample batch) at a time. Here every prompt x sample of an eval is submitted
in chunks of a few scheduler batches, so the continuous-batching scheduler
keeps ``max_batch_size`` sequences decoding on the GPU while earlier ones
finish.
"""

from __future__ import annotations

from typing import List, Sequence


def create_engine(param_path: str, batch_size: int, device=None, dtype=None, max_seq_len=None):
    from astrai_b200.eval.common import load_model
    from astrai_b200.inference import InferenceEngine

    model, tok = load_model(param_path, device, dtype)
    return InferenceEngine(model, tok, max_batch_size=batch_size, max_seq_len=max_seq_len), tok


def generate_many(engine, prompts: Sequence[str], max_tokens: int, temperature: float, top_p: float, top_k: int,
                  chunk: int = 0) -> List[str]:
    """Completions for every prompt, in order."""
    chunk = chunk or 4 * max(1, getattr(engine.scheduler, "max_batch_size", 1))
    out: List[str] = []
    for i in range(0, len(prompts), chunk):
        part = list(prompts[i:i + chunk])
        res = engine.generate(prompt=part, stream=False, max_tokens=max_tokens, temperature=temperature,
                              top_p=top_p, top_k=top_k)
        out.extend(res if isinstance(res, list) else [res])
    return out
