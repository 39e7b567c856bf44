"""Inference benchmark: prefill and decode throughput, contiguous or paged cache.

    python -m astrai_b200.cli.benchmark [--cache contiguous|paged] [--batch_size 4] [--prompt_length 512]
                                        [--gen_length 128] [--num_trials 5] [--prefill_only|--decode_only]

Parity: scripts/tools/benchmark.py:22-299 of the reference (same flags and
the same two measurements: a cache-less prefill forward, and a token-by-token
decode loop through the model with a bound cache view after a cached
prefill). Added: ``--engine`` also times the serving decode step (the
executor's CUDA-graph replay + fused sampling), and ``--reference_config``
selects the reference script's model (hidden 1536, 24 heads of 64); the
default is the 1.1B training config (heads of 128, the kernels' head size).
Times are CUDA events on the launching stream; one JSON line per result.
"""

from __future__ import annotations

import argparse
import json
from typing import List, Optional

import torch


def _config(reference: bool):
    from astrai_b200.config import AutoRegressiveLMConfig

    if reference:
        return AutoRegressiveLMConfig(vocab_size=10000, hidden_size=1536, num_attention_heads=24, num_key_value_heads=4,
                                      intermediate_size=6912, max_position_embeddings=2048, num_hidden_layers=24,
                                      rms_norm_eps=1e-5)
    return AutoRegressiveLMConfig(vocab_size=32000, hidden_size=2048, num_attention_heads=16, num_key_value_heads=4,
                                  intermediate_size=5632, max_position_embeddings=4096, num_hidden_layers=24,
                                  rms_norm_eps=1e-5, rope_theta=1e6)


def _make_cache(cfg, kind: str, batch: int, max_seq: int, device, dtype):
    from astrai_b200.inference import ContiguousCache, PageCache

    hd = cfg.hidden_size // cfg.num_attention_heads
    if kind == "contiguous":
        return ContiguousCache(cfg.num_hidden_layers, batch, max_seq, cfg.num_key_value_heads, hd, device, dtype)
    page = 128
    return PageCache(cfg.num_hidden_layers, -(-max_seq // page) * batch, page, cfg.num_key_value_heads, hd, device,
                     dtype)


def _timed(fn) -> float:
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / 1e3


@torch.inference_mode()
def run_prefill(model, cfg, batch: int, prompt: int, trials: int) -> dict:
    dev = next(model.parameters()).device
    for _ in range(3):
        model(torch.randint(0, cfg.vocab_size, (batch, prompt), device=dev))
    t = 0.0
    for _ in range(trials):
        ids = torch.randint(0, cfg.vocab_size, (batch, prompt), device=dev)
        t += _timed(lambda: model(ids))
    n = batch * prompt * trials
    return {"benchmark_type": "prefill", "tokens": n, "seconds": round(t, 4), "tokens_per_second": round(n / t, 1),
            "batch_size": batch, "prompt_length": prompt}


@torch.inference_mode()
def run_decode(model, cfg, kind: str, batch: int, prompt: int, gen: int, trials: int) -> dict:
    dev = next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    max_seq = prompt + gen
    t = 0.0
    for _ in range(trials + 1):  # the first trial warms up
        cache = _make_cache(cfg, kind, batch, max_seq, dev, dtype)
        tids = [f"b{i}" for i in range(batch)]
        for tid in tids:
            cache.task_alloc(tid, [0] * prompt)
            cache.task_extend(tid, max_seq - 1)
        ids = torch.randint(0, cfg.vocab_size, (batch, prompt), device=dev)
        gen_ids = torch.randint(0, cfg.vocab_size, (batch, gen), device=dev)
        pos = torch.arange(prompt, device=dev).unsqueeze(0).expand(batch, -1)
        model(ids, paged_cache=cache.bind(tids, [prompt] * batch, prompt, dev, uniform_start=0), position_ids=pos,
              logits_to_keep=1)

        def loop():
            for i in range(gen):
                p = prompt + i
                view = cache.bind(tids, [p + 1] * batch, 1, dev)
                model(gen_ids[:, i:i + 1], paged_cache=view,
                      position_ids=torch.full((batch, 1), p, device=dev, dtype=torch.long), logits_to_keep=1)

        dt = _timed(loop)
        if _ > 0 or trials == 0:
            t += dt
        for tid in tids:
            cache.task_free(tid)
    n = batch * gen * max(trials, 1)
    return {"benchmark_type": "decoding", "tokens": n, "seconds": round(t, 4), "tokens_per_second": round(n / t, 1),
            "batch_size": batch, "prompt_length": prompt, "gen_length": gen, "cache": kind, "path": "model loop"}


@torch.inference_mode()
def run_engine_decode(model, cfg, kind: str, batch: int, prompt: int, gen: int) -> dict:
    """Serving path: prefill + gen decode steps through the executor (CUDA graphs, fused sampling)."""
    from astrai_b200.inference.core.executor import Executor
    from astrai_b200.inference.core.task import Task

    dev = next(model.parameters()).device
    dtype = next(model.parameters()).dtype
    warm = 3
    max_seq = prompt + 1 + warm + gen  # prefill token + warm-up steps + timed steps
    cache = _make_cache(cfg, kind, batch, max_seq, dev, dtype)
    ex = Executor(model, None, cache, dev, dtype, use_cuda_graph=True, max_batch_size=batch, max_seq_len=max_seq,
                  seed=0)
    g = torch.Generator().manual_seed(0)
    tasks = [Task(f"t{i}", torch.randint(0, cfg.vocab_size, (prompt,), generator=g).tolist(), gen + 1,
                  temperature=0.8, top_p=0.95, top_k=50) for i in range(batch)]
    for t in tasks:
        cache.task_alloc(t.task_id, t.prompt_ids)
        cache.task_extend(t.task_id, max_seq - 1)
    ex.execute_prefill(tasks, prompt, 0)
    for _ in range(warm):  # capture + warm the graph
        ex.execute_decode(tasks)
    t = _timed(lambda: [ex.execute_decode(tasks) for _ in range(gen)])
    n = batch * gen
    return {"benchmark_type": "decoding", "tokens": n, "seconds": round(t, 4), "tokens_per_second": round(n / t, 1),
            "batch_size": batch, "prompt_length": prompt, "gen_length": gen, "cache": kind,
            "path": "executor (CUDA graph + fused sampling, host round trip per token)"}


def main(argv: Optional[List[str]] = None) -> None:
    from astrai_b200.models import AutoRegressiveLM

    p = argparse.ArgumentParser(description="AutoRegressiveLM inference benchmark")
    p.add_argument("--device", type=str, default="cuda")
    p.add_argument("--dtype", type=str, default="bfloat16", choices=["bfloat16", "float16", "float32"])
    p.add_argument("--cache", type=str, default="contiguous", choices=["contiguous", "paged"])
    p.add_argument("--batch_size", type=int, default=4)
    p.add_argument("--prompt_length", type=int, default=512)
    p.add_argument("--gen_length", type=int, default=128)
    p.add_argument("--num_trials", type=int, default=5)
    p.add_argument("--prefill_only", action="store_true")
    p.add_argument("--decode_only", action="store_true")
    p.add_argument("--engine", action="store_true", help="also time the serving decode step")
    p.add_argument("--reference_config", action="store_true", help="the reference script's model config")
    a = p.parse_args(argv)
    dtype = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[a.dtype]
    cfg = _config(a.reference_config)
    torch.manual_seed(0)
    with torch.device(a.device):
        model = AutoRegressiveLM(cfg).to(dtype=dtype).eval()
    if not a.decode_only:
        print(json.dumps(run_prefill(model, cfg, a.batch_size, a.prompt_length, a.num_trials)), flush=True)
    if not a.prefill_only:
        print(json.dumps(run_decode(model, cfg, a.cache, a.batch_size, a.prompt_length, a.gen_length,
                                    a.num_trials)), flush=True)
        if a.engine:
            print(json.dumps(run_engine_decode(model, cfg, a.cache, a.batch_size, a.prompt_length, a.gen_length)),
                  flush=True)


if __name__ == "__main__":
    main()
