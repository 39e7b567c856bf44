"""Inference engine facade.

Parity: astrai/inference/engine.py:16-348 (``GenerateResult``,
``GenerationRequest`` with the same validation, ``InferenceEngine`` with
``generate`` (str or list, streaming or not), ``generate_async``,
``generate_with_request``, ``get_stats``, ``shutdown`` and context-manager
use). ``page_size`` builds a :class:`PageCache` (prefix sharing) instead of
the per-slot cache when ``n_pages`` is given.
"""

from __future__ import annotations

import asyncio
import gc
import threading
from typing import Any, AsyncGenerator, Dict, Generator, List, Optional, Tuple, Union

import torch
import torch.nn as nn

from astrai_b200.inference.core.cache import KVCache, PageCache
from astrai_b200.inference.core.scheduler import InferenceScheduler, model_head_dim
from astrai_b200.inference.core.task import STOP


class GenerateResult:
    """Thread-safe collector of streamed pieces for ``count`` prompts."""

    def __init__(self, count: int = 1):
        self._cond = threading.Condition()
        self._event = threading.Event()
        self.tokens: List[Tuple[int, Any]] = []
        self.results: List[str] = [""] * count
        self._done = [False] * count
        self._completed = 0
        self._total = count

    def append(self, token, idx: int = 0) -> None:
        with self._cond:
            self.tokens.append((idx, token))
            if token is STOP:
                if not self._done[idx]:
                    self._done[idx] = True
                    self._completed += 1
                    self._cond.notify_all()
            else:
                self.results[idx] += token
            self._event.set()

    def pop_all(self) -> List[Tuple[int, Any]]:
        with self._cond:
            out, self.tokens = self.tokens, []
            if not out:
                self._event.clear()
            return out

    def wait(self, timeout: Optional[float] = None) -> bool:
        return self._event.wait(timeout=timeout)

    def wait_completion(self, timeout: float = 300.0) -> None:
        with self._cond:
            if not self._cond.wait_for(lambda: self._completed >= self._total, timeout=timeout):
                raise TimeoutError(f"Generation timeout after {timeout}s ({self._completed}/{self._total} completed)")

    def get_results(self) -> List[str]:
        with self._cond:
            return list(self.results)


class GenerationRequest:
    """Chat request with validated sampling parameters."""

    def __init__(self, messages: List[Dict[str, str]], top_k: int = 50, top_p: float = 1.0,
                 temperature: float = 1.0, max_tokens: Optional[int] = None, frequency_penalty: float = 0.0,
                 rep_window: int = 64, stream: bool = False):
        if not (isinstance(top_k, int) and top_k >= 0):
            raise ValueError("top_k must be a non-negative integer")
        if not (0.0 <= top_p <= 1.0):
            raise ValueError("top_p must be a float between 0.0 and 1.0")
        if not (isinstance(temperature, (int, float)) and temperature >= 0):
            raise ValueError("temperature must be a non-negative number")
        if not (isinstance(frequency_penalty, (int, float)) and -2.0 <= frequency_penalty <= 2.0):
            raise ValueError("frequency_penalty must be between -2.0 and 2.0")
        if not (isinstance(rep_window, int) and rep_window > 0):
            raise ValueError("rep_window must be a positive integer")
        self.messages = messages
        self.top_k, self.top_p, self.temperature = top_k, top_p, temperature
        self.max_tokens = max_tokens
        self.frequency_penalty, self.rep_window = frequency_penalty, rep_window
        self.stream = stream


class InferenceEngine:
    """Continuous-batching generation behind a simple API."""

    def __init__(self, model: nn.Module, tokenizer, max_batch_size: int = 1, max_seq_len: Optional[int] = None,
                 max_prompt_len: int = 2048, page_size: int = 128, cache: Optional[KVCache] = None,
                 n_pages: Optional[int] = None, use_cuda_graph: Optional[bool] = None, seed: Optional[int] = None):
        self.model = model
        self.tokenizer = tokenizer
        if cache is None and n_pages:
            p = next(model.parameters())
            cfg = model.config
            cache = PageCache(cfg.num_hidden_layers, n_pages, page_size, cfg.num_key_value_heads,
                              model_head_dim(model), p.device, p.dtype)
        self.scheduler = InferenceScheduler(model, tokenizer, max_batch_size=max_batch_size, max_seq_len=max_seq_len,
                                            max_prompt_len=max_prompt_len, cache=cache,
                                            use_cuda_graph=use_cuda_graph, seed=seed)
        self.scheduler.start()

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        self.shutdown()
        return False

    # ------------------------------------------------------------------ public API
    def generate(self, prompt: Union[str, List[str]], stream: bool = False, max_tokens: Optional[int] = None,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = 50, frequency_penalty: float = 0.0,
                 rep_window: int = 64) -> Union[Generator, str, List[str]]:
        batch = isinstance(prompt, list)
        prompts = prompt if batch else [prompt]
        params = dict(max_tokens=max_tokens, temperature=temperature, top_p=top_p, top_k=top_k,
                      frequency_penalty=frequency_penalty, rep_window=rep_window)
        if stream:
            return self._generate_streaming(prompts, batch, **params)
        return self._generate_blocking(prompts, batch, **params)

    def generate_async(self, prompt: str, max_tokens: Optional[int] = None, temperature: float = 1.0,
                       top_p: float = 1.0, top_k: int = 50, frequency_penalty: float = 0.0,
                       rep_window: int = 64) -> AsyncGenerator[str, None]:
        gen = self._generate_streaming([prompt], False, max_tokens=max_tokens, temperature=temperature, top_p=top_p,
                                       top_k=top_k, frequency_penalty=frequency_penalty, rep_window=rep_window)

        async def agen():
            loop = asyncio.get_running_loop()
            try:
                while True:
                    piece = await loop.run_in_executor(None, self._next_token, gen)
                    if piece is None:
                        break
                    yield piece
            finally:  # closing early (stop sequence, client gone) cancels the task
                gen.close()

        return agen()

    @staticmethod
    def _next_token(gen: Generator) -> Optional[str]:
        try:
            return next(gen)
        except StopIteration:
            return None

    def generate_with_request(self, request: GenerationRequest):
        prompt = self.tokenizer.apply_chat_template(request.messages, tokenize=False)
        return self.generate(prompt, stream=request.stream, max_tokens=request.max_tokens,
                             temperature=request.temperature, top_p=request.top_p, top_k=request.top_k,
                             frequency_penalty=request.frequency_penalty, rep_window=request.rep_window)

    def get_stats(self) -> Dict[str, Any]:
        return self.scheduler.get_stats()

    def shutdown(self) -> None:
        self.scheduler.stop()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        gc.collect()

    # ------------------------------------------------------------------ internals
    def _submit(self, prompts: List[str], **params) -> Tuple[GenerateResult, List[str]]:
        result = GenerateResult(len(prompts))
        ids = []
        for i, p in enumerate(prompts):
            ids.append(self.scheduler.add_task(p, stream_callback=(lambda tok, i=i: result.append(tok, i)), **params))
        return result, ids

    def _generate_streaming(self, prompts: List[str], batch: bool, **params) -> Generator:
        result, task_ids = self._submit(prompts, **params)
        n = len(prompts)

        def gen():
            done = [False] * n
            left = n
            try:
                while left:
                    for idx, tok in result.pop_all():
                        if tok is STOP:
                            if not done[idx]:
                                done[idx] = True
                                left -= 1
                        else:
                            yield (idx, tok) if batch else tok
                    if left:
                        result.wait(timeout=0.05)
            finally:
                for tid in task_ids:
                    self.scheduler.remove_task(tid)

        return gen()

    def _generate_blocking(self, prompts: List[str], batch: bool, **params) -> Union[str, List[str]]:
        result, task_ids = self._submit(prompts, **params)
        try:
            result.wait_completion()
        finally:
            for tid in task_ids:
                self.scheduler.remove_task(tid)
        res = result.get_results()
        return res if batch else res[0]
