"""Prefill / decode steps of the inference loop.

Parity: astrai/inference/core/executor.py:15-166 (``Executor`` with
``execute_prefill(tasks, prompt_len, start_pos)`` and
``execute_decode(tasks, return_logprobs)``).

Differences, all on the device side:

* no dense masks are built: the cache view knows each row's length and the
  kernels apply causality themselves;
* prefill keeps only the last position's logits (``logits_to_keep=1``) and
  samples each task's first token from them;
* a decode step's host inputs (ids, positions, lengths, page table, sampling
  parameters) are packed into three pinned staging buffers and copied with
  three H2D copies; with ``use_cuda_graph`` the whole decode forward +
  sampling for a batch-size bucket is replayed from a captured CUDA graph
  (rows whose frequency penalty is non-zero take the eager path, which also
  ships the history window).
"""

from __future__ import annotations

import logging
from typing import Dict, List, Optional, Tuple

import torch

from astrai_b200.inference.core.cache import KVCache, PageCacheView
from astrai_b200.inference.core.task import Task
from astrai_b200.inference.sample import DeviceRNG, fused_sample, sample

logger = logging.getLogger(__name__)

_BUCKETS = (1, 2, 4, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256)


def _bucket(n: int, cap: int) -> int:
    for b in _BUCKETS:
        if b >= n:
            return min(b, cap)
    return cap


class _DecodeGraphs:
    """Static decode inputs + one captured graph per batch-size bucket."""

    def __init__(self, executor: "Executor", max_batch: int, max_pages: int):
        self.ex = executor
        dev = executor.device
        self.max_batch, self.max_pages = max_batch, max_pages
        B, P = max_batch, max_pages
        # int64: ids, positions; int32: pos32, lens, top_k, table; fp32: temperature, top_p, penalty
        self.i64 = torch.zeros(2 * B, dtype=torch.int64, device=dev)
        self.i32 = torch.zeros(B * (3 + P), dtype=torch.int32, device=dev)
        self.f32 = torch.zeros(3 * B, dtype=torch.float32, device=dev)
        self.h_i64 = torch.zeros(2 * B, dtype=torch.int64).pin_memory()
        self.h_i32 = torch.zeros(B * (3 + P), dtype=torch.int32).pin_memory()
        self.h_f32 = torch.zeros(3 * B, dtype=torch.float32).pin_memory()
        self.out_tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.out_lp = torch.zeros(B, dtype=torch.float32, device=dev)
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.pool = None

    def _views(self, b: int):
        B, P = self.max_batch, self.max_pages
        ids = self.i64[:B].view(B, 1)[:b]
        pos = self.i64[B:].view(B, 1)[:b]
        pos32 = self.i32[:B][:b]
        lens = self.i32[B:2 * B][:b]
        topk = self.i32[2 * B:3 * B][:b]
        table = self.i32[3 * B:].view(B, P)[:b]
        temp, topp, pen = (self.f32[i * B:(i + 1) * B][:b] for i in range(3))
        return ids, pos, pos32, lens, topk, table, temp, topp, pen

    def stage(self, tasks: List[Task]) -> int:
        ex, B, P = self.ex, self.max_batch, self.max_pages
        n = len(tasks)
        b = _bucket(n, B)
        hi, h32, hf = self.h_i64.numpy(), self.h_i32.numpy(), self.h_f32.numpy()  # share the pinned memory
        tables = ex.kv_cache._table  # noqa: SLF001 - executor and cache are one subsystem
        table = h32[3 * B:].reshape(B, P)
        table[:b] = -1
        hi[:b] = 0
        hi[B:B + b] = 0
        h32[:b] = 0
        h32[B:B + b] = 0
        h32[2 * B:2 * B + b] = 0
        hf[:b], hf[B:B + b], hf[2 * B:2 * B + b] = 0.0, 1.0, 0.0  # padding rows: no keys, no write, greedy
        for r, t in enumerate(tasks):
            pos = t.next_pos
            hi[r] = t.output_ids[-1]
            hi[B + r] = pos
            h32[r] = pos
            h32[B + r] = pos + 1
            h32[2 * B + r] = t.top_k
            pages = tables.get(t.task_id)
            table[r, : len(pages)] = pages
            hf[r], hf[B + r], hf[2 * B + r] = t.temperature, t.top_p, t.frequency_penalty
        self.i64.copy_(self.h_i64, non_blocking=True)
        self.i32.copy_(self.h_i32, non_blocking=True)
        self.f32.copy_(self.h_f32, non_blocking=True)
        return b

    def _forward(self, b: int):
        ex = self.ex
        ids, pos, pos32, lens, topk, table, temp, topp, pen = self._views(b)
        view = PageCacheView(ex.kv_cache.storage, table, lens=lens, n_new=1, positions=pos32,
                             workspace=self.workspace(b), splits=self.splits(b))
        out = ex.model(ids, position_ids=pos, paged_cache=view, logits_to_keep=1)
        fused_sample(out["logits"][:, -1], temp, topk, topp, pen, None, ex.rng, self.out_tok[:b], self.out_lp[:b])

    def splits(self, b: int) -> int:
        from astrai_b200.ops._ext import native

        st = self.ex.kv_cache.storage
        return int(native().decode_splits(b, st.n_kv_heads, self.max_pages * st.page_size,
                                          self.ex.device.index or 0))

    def workspace(self, b: int):
        if not hasattr(self, "_ws"):
            n_heads = self.ex.n_heads
            self._ws = torch.empty(self.max_batch * n_heads * 64 * 130, dtype=torch.float32, device=self.ex.device)
        return self._ws

    def run(self, tasks: List[Task]) -> Tuple[List[int], List[float]]:
        b = self.stage(tasks)
        g = self.graphs.get(b)
        if g is None:
            s = torch.cuda.Stream(device=self.ex.device)
            s.wait_stream(torch.cuda.current_stream(self.ex.device))
            with torch.cuda.stream(s), torch.inference_mode():
                self._forward(b)  # warm-up: kernel attributes, tensor maps, allocator
            torch.cuda.current_stream(self.ex.device).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.inference_mode(), torch.cuda.graph(g, pool=self.pool):
                self._forward(b)
            self.pool = g.pool()
            self.graphs[b] = g
        g.replay()
        n = len(tasks)
        return self.out_tok[:n].tolist(), self.out_lp[:n].tolist()


class Executor:
    """Model forward passes for prefill and decode."""

    def __init__(self, model, tokenizer, kv_cache: KVCache, device=None, dtype: Optional[torch.dtype] = None,
                 use_cuda_graph: bool = False, max_batch_size: int = 16, max_seq_len: int = 2048,
                 seed: Optional[int] = None):
        self.model = model
        self.tokenizer = tokenizer
        self.kv_cache = kv_cache
        p = next(model.parameters())
        self.device = torch.device(device) if device is not None else p.device
        self.dtype = dtype or p.dtype
        cfg = model.config
        self.n_heads = cfg.num_attention_heads
        self.rng = DeviceRNG(self.device, seed) if self.device.type == "cuda" else None
        self._cpu_gen = torch.Generator().manual_seed(seed) if seed is not None else None
        self._graphs: Optional[_DecodeGraphs] = None
        if use_cuda_graph and self.device.type == "cuda":
            page = getattr(kv_cache, "page_size", max_seq_len)
            self._graphs = _DecodeGraphs(self, max_batch_size, -(-max_seq_len // page))

    # ----------------------------------------------------------------- helpers
    def _sample(self, logits: torch.Tensor, tasks: List[Task]) -> Tuple[List[int], List[float]]:
        dev = logits.device
        n = len(tasks)
        pen_on = any(t.frequency_penalty != 0.0 for t in tasks)
        hist = None
        if pen_on:
            rows = [t.history() for t in tasks]
            w = max(len(r) for r in rows)
            hist = torch.full((n, max(w, 1)), -1, dtype=torch.int64)
            for i, r in enumerate(rows):
                hist[i, : len(r)] = torch.tensor(r, dtype=torch.int64)
        if dev.type == "cuda" and self.rng is not None:
            f = torch.tensor([[t.temperature, t.top_p, t.frequency_penalty] for t in tasks],
                             dtype=torch.float32).to(dev, non_blocking=True)
            k = torch.tensor([t.top_k for t in tasks], dtype=torch.int32).to(dev, non_blocking=True)
            tok = torch.empty(n, dtype=torch.int64, device=dev)
            lp = torch.empty(n, dtype=torch.float32, device=dev)
            fused_sample(logits.contiguous() if logits.stride(-1) != 1 else logits, f[:, 0].contiguous(), k,
                         f[:, 1].contiguous(), f[:, 2].contiguous(),
                         hist.to(dev, non_blocking=True) if hist is not None else None, self.rng, tok, lp)
            return tok.tolist(), lp.tolist()
        tok, lp = sample(logits.float(), temperature=torch.tensor([t.temperature for t in tasks]),
                         top_k=torch.tensor([t.top_k for t in tasks]), top_p=torch.tensor([t.top_p for t in tasks]),
                         frequency_penalty=torch.tensor([t.frequency_penalty for t in tasks]),
                         input_ids=hist, input_mask=(hist >= 0) if hist is not None else None, return_logprobs=True)
        return tok.tolist(), lp.tolist()

    # ----------------------------------------------------------------- steps
    @torch.inference_mode()
    def execute_prefill(self, tasks: List[Task], prompt_len: int, start_pos: int = 0,
                        return_logprobs: bool = False) -> List:
        """Prefill ``prompt_ids[start_pos:prompt_len]`` of equal-length tasks and
        sample each task's first token (appended to ``task.output_ids``)."""
        if not tasks:
            return []
        dev = self.device
        S = prompt_len - start_pos
        ids = torch.tensor([t.prompt_ids[start_pos:prompt_len] for t in tasks], dtype=torch.long)
        ids = ids.to(dev, non_blocking=True)
        pos = torch.arange(start_pos, prompt_len, device=dev).unsqueeze(0).expand(len(tasks), -1)
        view = self.kv_cache.bind([t.task_id for t in tasks], [prompt_len] * len(tasks), S, dev,
                                  uniform_start=start_pos)
        logits = self.model(ids, position_ids=pos, paged_cache=view, logits_to_keep=1)["logits"][:, -1]
        toks, lps = self._sample(logits, tasks)
        return self._append(tasks, toks, lps, return_logprobs)

    @torch.inference_mode()
    def execute_decode(self, tasks: List[Task], return_logprobs: bool = False) -> List:
        """One token for every task (fed: its last output token)."""
        if not tasks:
            return []
        if self._graphs is not None and len(tasks) <= self._graphs.max_batch and not any(
                t.frequency_penalty != 0.0 for t in tasks):
            toks, lps = self._graphs.run(tasks)
            return self._append(tasks, toks, lps, return_logprobs)
        dev = self.device
        ids = torch.tensor([[t.output_ids[-1]] for t in tasks], dtype=torch.long).to(dev, non_blocking=True)
        positions = [t.next_pos for t in tasks]
        pos = torch.tensor(positions, dtype=torch.long).to(dev, non_blocking=True)
        view = self.kv_cache.bind([t.task_id for t in tasks], [p + 1 for p in positions], 1, dev)
        logits = self.model(ids, position_ids=pos.unsqueeze(1), paged_cache=view, logits_to_keep=1)["logits"][:, -1]
        toks, lps = self._sample(logits, tasks)
        return self._append(tasks, toks, lps, return_logprobs)

    @staticmethod
    def _append(tasks: List[Task], toks: List[int], lps: List[float], return_logprobs: bool) -> List:
        for t, tok, lp in zip(tasks, toks, lps):
            t.output_ids.append(int(tok))
            t.output_logprobs.append(float(lp))
            t.output_tokens += 1
        return list(zip(toks, lps)) if return_logprobs else list(toks)
