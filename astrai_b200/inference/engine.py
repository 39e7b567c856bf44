"""Inference engine: the user-facing generation API over the continuous-batching scheduler.

Public surface kept from the reference (astrai/inference/engine.py:17-348): ``GenerateResult``,
``GenerationRequest``, and ``InferenceEngine`` with ``generate`` (one prompt or a list, streamed
or blocking), ``generate_async``, ``generate_with_request``, ``get_stats``, ``shutdown`` and
context-manager use.

Design: every call submits its prompts as scheduler tasks whose stream callbacks push
``(prompt index, piece)`` events into one FIFO owned by the call (:class:`GenerateResult`). The
scheduler thread only enqueues; the caller's thread is the only consumer. Blocking and streaming
generation are the same drain loop (:meth:`GenerateResult.events`); the blocking form just joins
the pieces. The end of a prompt's stream is the ``STOP`` sentinel. Leaving a drain loop early
(a consumer that stops iterating, a timeout) removes the call's tasks from the scheduler, so
their KV pages come back. With ``n_pages`` set, the engine builds a :class:`PageCache` (prefix
sharing across requests) instead of the per-slot contiguous cache.
"""

from __future__ import annotations

import asyncio
import gc
import queue
import time
from typing import Any, AsyncIterator, Dict, Iterator, List, Optional, Sequence, Tuple, Union

import torch
import torch.nn as nn

from astrai_b200.inference.core.cache import KVCache, PageCache
from astrai_b200.inference.core.scheduler import InferenceScheduler, model_head_dim
from astrai_b200.inference.core.task import STOP

_POLL_S = 0.05  # how often a blocked consumer re-checks its deadline


class GenerateResult:
    """Event FIFO for one generation call over ``count`` prompts.

    ``append(piece, idx)`` is the scheduler-side callback (thread-safe, never blocks).
    ``events(timeout)`` yields ``(idx, piece)`` in arrival order until every prompt has
    delivered ``STOP``; the pieces are also kept so ``get_results()`` returns the full texts.
    """

    def __init__(self, count: int = 1):
        self._fifo: "queue.SimpleQueue[Tuple[int, Any]]" = queue.SimpleQueue()
        self._pieces: List[List[str]] = [[] for _ in range(count)]
        self._open = set(range(count))

    # producer side (scheduler thread)
    def append(self, token: Any, idx: int = 0) -> None:
        self._fifo.put((idx, token))

    # consumer side (the calling thread)
    @property
    def finished(self) -> bool:
        return not self._open

    def events(self, timeout: Optional[float] = None) -> Iterator[Tuple[int, str]]:
        """Drain the FIFO until every prompt is finished. ``timeout`` bounds the silence between
        two events (None: wait for ever); on expiry a ``TimeoutError`` names the open prompts."""
        last = time.monotonic()
        while self._open:
            try:
                idx, piece = self._fifo.get(timeout=_POLL_S)
            except queue.Empty:
                if timeout is not None and time.monotonic() - last > timeout:
                    raise TimeoutError(f"no output for {timeout:.0f} s; prompts still running: "
                                       f"{sorted(self._open)} of {len(self._pieces)}") from None
                continue
            last = time.monotonic()
            if piece is STOP:
                self._open.discard(idx)
                continue
            self._pieces[idx].append(piece)
            yield idx, piece

    def get_results(self) -> List[str]:
        return ["".join(p) for p in self._pieces]


def _check_sampling(top_k, top_p, temperature, frequency_penalty, rep_window) -> None:
    problems = []
    if not isinstance(top_k, int) or isinstance(top_k, bool) or top_k < 0:
        problems.append(f"top_k={top_k!r} (want an int >= 0; 0 disables the cut)")
    if not isinstance(top_p, (int, float)) or not 0.0 <= top_p <= 1.0:
        problems.append(f"top_p={top_p!r} (want a number in [0, 1])")
    if not isinstance(temperature, (int, float)) or temperature < 0:
        problems.append(f"temperature={temperature!r} (want a number >= 0; 0 is greedy)")
    if not isinstance(frequency_penalty, (int, float)) or abs(frequency_penalty) > 2.0:
        problems.append(f"frequency_penalty={frequency_penalty!r} (want a number in [-2, 2])")
    if not isinstance(rep_window, int) or rep_window <= 0:
        problems.append(f"rep_window={rep_window!r} (want an int > 0)")
    if problems:
        raise ValueError("invalid sampling parameters: " + "; ".join(problems))


class GenerationRequest:
    """A chat-formatted request (``messages`` in the tokenizer's chat-template format) with its
    sampling parameters, validated on construction (``ValueError`` lists every bad field)."""

    def __init__(self, messages: List[Dict[str, str]], top_k: int = 50, top_p: float = 1.0,
                 temperature: float = 1.0, max_tokens: Optional[int] = None, frequency_penalty: float = 0.0,
                 rep_window: int = 64, stream: bool = False):
        _check_sampling(top_k, top_p, temperature, frequency_penalty, rep_window)
        self.messages = messages
        self.top_k = top_k
        self.top_p = top_p
        self.temperature = temperature
        self.max_tokens = max_tokens
        self.frequency_penalty = frequency_penalty
        self.rep_window = rep_window
        self.stream = stream

    def sampling(self) -> Dict[str, Any]:
        return {"max_tokens": self.max_tokens, "temperature": self.temperature, "top_p": self.top_p,
                "top_k": self.top_k, "frequency_penalty": self.frequency_penalty, "rep_window": self.rep_window}


def _text_only(events: Iterator[Tuple[int, str]]) -> Iterator[str]:
    try:
        for _, piece in events:
            yield piece
    finally:
        events.close()  # release the tasks now, not when the garbage collector gets to it


class InferenceEngine:
    """Generation front end. The scheduler thread starts with the engine and stops in
    :meth:`shutdown` (or on leaving a ``with`` block)."""

    #: seconds without any output after which a blocking call gives up
    timeout_s: float = 300.0

    def __init__(self, model: nn.Module, tokenizer, max_batch_size: int = 1, max_seq_len: Optional[int] = None,
                 max_prompt_len: int = 2048, page_size: int = 128, cache: Optional[KVCache] = None,
                 n_pages: Optional[int] = None, use_cuda_graph: Optional[bool] = None, seed: Optional[int] = None):
        self.model = model
        self.tokenizer = tokenizer
        if cache is None and n_pages:
            cache = self._paged_cache(model, n_pages, page_size)
        self.scheduler = InferenceScheduler(model, tokenizer, max_batch_size=max_batch_size, max_seq_len=max_seq_len,
                                            max_prompt_len=max_prompt_len, cache=cache,
                                            use_cuda_graph=use_cuda_graph, seed=seed)
        self.scheduler.start()

    @staticmethod
    def _paged_cache(model: nn.Module, n_pages: int, page_size: int) -> PageCache:
        ref = next(model.parameters())
        c = model.config
        return PageCache(c.num_hidden_layers, n_pages, page_size, c.num_key_value_heads, model_head_dim(model),
                         ref.device, ref.dtype)

    def __enter__(self) -> "InferenceEngine":
        return self

    def __exit__(self, *exc) -> bool:
        self.shutdown()
        return False

    # ------------------------------------------------------------------ submission
    def _launch(self, prompts: Sequence[str], sampling: Dict[str, Any]) -> Tuple[GenerateResult, List[str]]:
        res = GenerateResult(len(prompts))
        tasks = [self.scheduler.add_task(text, stream_callback=lambda piece, i=i: res.append(piece, i), **sampling)
                 for i, text in enumerate(prompts)]
        return res, tasks

    def _release(self, tasks: Sequence[str]) -> None:
        for t in tasks:
            self.scheduler.remove_task(t)

    def _drain(self, prompts: Sequence[str], sampling: Dict[str, Any],
               timeout: Optional[float]) -> Iterator[Tuple[int, str]]:
        """(idx, piece) events of a fresh call; the tasks are released however the loop ends."""
        res, tasks = self._launch(prompts, sampling)
        try:
            yield from res.events(timeout)
        finally:
            self._release(tasks)

    # ------------------------------------------------------------------ public API
    def generate(self, prompt: Union[str, List[str]], stream: bool = False, max_tokens: Optional[int] = None,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = 50, frequency_penalty: float = 0.0,
                 rep_window: int = 64) -> Union[Iterator, str, List[str]]:
        """Blocking: the generated text (a list of texts for a list of prompts). Streaming: an
        iterator of text pieces (of ``(prompt index, piece)`` pairs for a list of prompts)."""
        as_list = isinstance(prompt, list)
        prompts = prompt if as_list else [prompt]
        sampling = {"max_tokens": max_tokens, "temperature": temperature, "top_p": top_p, "top_k": top_k,
                    "frequency_penalty": frequency_penalty, "rep_window": rep_window}
        if stream:
            events = self._drain(prompts, sampling, None)
            return events if as_list else _text_only(events)
        texts: List[List[str]] = [[] for _ in prompts]
        for i, piece in self._drain(prompts, sampling, self.timeout_s):
            texts[i].append(piece)
        out = ["".join(t) for t in texts]
        return out if as_list else out[0]

    def generate_async(self, prompt: str, max_tokens: Optional[int] = None, temperature: float = 1.0,
                       top_p: float = 1.0, top_k: int = 50, frequency_penalty: float = 0.0,
                       rep_window: int = 64) -> AsyncIterator[str]:
        """Async iterator of text pieces for one prompt. The blocking queue reads run in the event
        loop's default executor; closing the iterator early cancels the task."""
        pieces = self.generate(prompt, stream=True, max_tokens=max_tokens, temperature=temperature, top_p=top_p,
                               top_k=top_k, frequency_penalty=frequency_penalty, rep_window=rep_window)
        end = object()

        def pull():
            return next(pieces, end)

        async def stream():
            loop = asyncio.get_running_loop()
            try:
                while (piece := await loop.run_in_executor(None, pull)) is not end:
                    yield piece
            finally:
                pieces.close()

        return stream()

    def generate_with_request(self, request: GenerationRequest):
        """Render ``request.messages`` with the tokenizer's chat template, then :meth:`generate`."""
        text = self.tokenizer.apply_chat_template(request.messages, tokenize=False)
        return self.generate(text, stream=request.stream, **request.sampling())

    def get_stats(self) -> Dict[str, Any]:
        return self.scheduler.get_stats()

    def shutdown(self) -> None:
        """Stop the scheduler thread and hand cached device memory back."""
        self.scheduler.stop()
        gc.collect()
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
