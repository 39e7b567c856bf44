"""Continuous-batching scheduler.

Parity: astrai/inference/core/scheduler.py:17-311 (``InferenceScheduler``:
``add_task``, ``remove_task``, ``get_stats``, ``start``, ``stop``, the daemon
loop cleanup -> refill -> prefill grouped by (prompt length, cached length)
-> one batched decode step for every running task -> stream callbacks, and
the synchronous ``run_batch`` used for RL rollouts).

The loop runs its forward passes through :class:`Executor`; the decode step
replays a captured CUDA graph per batch-size bucket when ``use_cuda_graph``
(default on CUDA), so a step costs three small H2D copies, one graph launch
and one D2H read of the sampled tokens.
"""

from __future__ import annotations

import logging
import threading
import uuid
from typing import Any, Dict, List, Optional, Tuple

import torch

from astrai_b200.inference.core.cache import ContiguousCache, KVCache
from astrai_b200.inference.core.executor import Executor
from astrai_b200.inference.core.task import STOP, Task, TaskManager, TaskStatus

logger = logging.getLogger(__name__)


def model_head_dim(model) -> int:
    cfg = model.config
    if getattr(cfg, "attn_type", "gqa") == "mla":
        return int(cfg.qk_nope_head_dim) + int(cfg.qk_rope_head_dim)
    return cfg.hidden_size // cfg.num_attention_heads


class InferenceScheduler:
    def __init__(self, model, tokenizer, max_batch_size: int = 16, max_seq_len: Optional[int] = None,
                 max_prompt_len: int = 2048, device=None, dtype: Optional[torch.dtype] = None,
                 cache: Optional[KVCache] = None, use_cuda_graph: Optional[bool] = None, seed: Optional[int] = None):
        cfg = model.config
        if max_seq_len is None:
            max_seq_len = getattr(cfg, "max_position_embeddings", None)
            if max_seq_len is None:
                raise ValueError("max_seq_len must be given or set as config.max_position_embeddings")
        self.max_seq_len = int(max_seq_len)
        self.max_batch_size = int(max_batch_size)
        p = next(model.parameters())
        self.model = model
        self.device = torch.device(device) if device is not None else p.device
        self.dtype = dtype or p.dtype
        self._cache = cache if cache is not None else ContiguousCache(
            cfg.num_hidden_layers, max_batch_size, self.max_seq_len, cfg.num_key_value_heads, model_head_dim(model),
            self.device, self.dtype)
        self._task_mgr = TaskManager(tokenizer, max_batch_size, self.max_seq_len, max_prompt_len)
        if use_cuda_graph is None:
            use_cuda_graph = self.device.type == "cuda" and self.dtype == torch.bfloat16
        self._executor = Executor(model, tokenizer, self._cache, self.device, self.dtype,
                                  use_cuda_graph=use_cuda_graph, max_batch_size=max_batch_size,
                                  max_seq_len=self.max_seq_len, seed=seed)
        self._stop_event = threading.Event()
        self._loop_thread: Optional[threading.Thread] = None
        self._step_lock = threading.RLock()

    @property
    def cache(self) -> KVCache:
        return self._cache

    @property
    def executor(self) -> Executor:
        return self._executor

    @property
    def tokenizer(self):
        return self._task_mgr.tokenizer

    # ------------------------------------------------------------------ task API
    def add_task(self, prompt: str, **kwargs) -> str:
        return self._task_mgr.add_task(prompt, **kwargs)

    def remove_task(self, task_id: str) -> None:
        with self._step_lock:  # never free pages under a running step
            for t in self._task_mgr.remove_task(task_id):
                self._cache.task_free(t.task_id)

    def get_stats(self) -> Dict[str, Any]:
        return self._task_mgr.get_stats()

    # ------------------------------------------------------------------ one iteration
    def _prefill(self, tasks: List[Task], return_logprobs: bool = False) -> None:
        groups: Dict[Tuple[int, int], List[Task]] = {}
        for t in tasks:
            t.input_tokens = len(t.prompt_ids)
            groups.setdefault((len(t.prompt_ids), self._cache.task_cached(t.task_id)), []).append(t)
        page = getattr(self._cache, "page_size", 64)
        for (plen, start), group in groups.items():
            self._executor.execute_prefill(group, plen, start, return_logprobs)
            for t in group:
                self._cache.task_record_hashes(t.task_id, t.prompt_ids, start // page)

    def _emit(self, tasks: List[Task], stop_ids) -> None:
        mgr = self._task_mgr
        for t in tasks:
            text = t.decode_new_token(mgr.tokenizer)
            if text:
                mgr.invoke_callback(t.task_id, text)
            if t.is_finished(stop_ids):
                rest = t.flush_remaining(mgr.tokenizer)
                if rest:
                    mgr.invoke_callback(t.task_id, rest)
                mgr.invoke_callback(t.task_id, STOP)

    def step(self) -> bool:
        """One scheduler iteration; False when there was nothing to do."""
        with self._step_lock:
            return self._step()

    def _step(self) -> bool:
        mgr, cache = self._task_mgr, self._cache
        stop_ids = mgr.tokenizer.stop_ids
        for t in mgr.remove_finished_tasks(stop_ids):
            cache.task_free(t.task_id)
        free = mgr.max_batch_size - len(mgr.get_active_tasks())
        if free > 0:
            failed = []
            for t in mgr.pull_candidates(free):
                (mgr.activate if cache.task_alloc(t.task_id, t.prompt_ids) else failed.append)(t)
            if failed:
                mgr.return_to_waiting(failed)
        if not mgr.has_work():
            return False
        fresh = [t for t in mgr.get_active_tasks() if not t.output_ids]
        if fresh:
            self._prefill(fresh)
            self._emit(fresh, stop_ids)
        running = [t for t in mgr.get_active_tasks() if t.output_ids and not t.is_finished(stop_ids)
                   and t.status == TaskStatus.RUNNING and t not in fresh]
        valid = []
        for t in sorted(running, key=lambda x: x.task_id):
            if cache.task_extend(t.task_id, t.next_pos):
                valid.append(t)
            else:
                t.status = TaskStatus.ABORTED
                mgr.invoke_callback(t.task_id, STOP)
        if valid:
            self._executor.execute_decode(valid)
            self._emit(valid, stop_ids)
        return True

    def _run_generation_loop(self) -> None:
        try:
            while not self._stop_event.is_set():
                if not self.step():
                    self._task_mgr.wait_for_tasks(timeout=1.0)
        except Exception as e:  # fail every request rather than leaving callers waiting
            self._stop_event.set()
            logger.error("Scheduler loop crashed: %s", e, exc_info=True)
            self._abort_all()

    def _abort_all(self) -> None:
        with self._step_lock:
            self._abort_all_locked()

    def _abort_all_locked(self) -> None:
        mgr = self._task_mgr
        for t in mgr.get_active_tasks():
            mgr.invoke_callback(t.task_id, STOP)
            self._cache.task_free(t.task_id)
        for t in mgr.get_waiting_tasks():
            mgr.invoke_callback(t.task_id, STOP)
        mgr.clear_queues()

    def start(self) -> None:
        if self._loop_thread is not None and self._loop_thread.is_alive():
            return
        self._stop_event.clear()
        self._loop_thread = threading.Thread(target=self._run_generation_loop, daemon=True)
        self._loop_thread.start()

    def stop(self) -> None:
        self._stop_event.set()
        self._task_mgr.wake()
        if self._loop_thread is not None:
            self._loop_thread.join(timeout=5.0)
        self._loop_thread = None
        self._abort_all()

    # ------------------------------------------------------------------ synchronous batch (RL rollout)
    def run_batch(self, prompt_ids_list: List[List[int]], *, max_tokens: Optional[int] = None,
                  temperature: float = 1.0, top_p: float = 1.0, top_k: int = 50, frequency_penalty: float = 0.0,
                  rep_window: int = 64, return_logprobs: bool = False) -> List[Any]:
        """Generate for already-tokenised prompts on the calling thread.

        Prompts run in waves of at most ``max_batch_size``; a prompt that does
        not fit ``max_seq_len`` (or the cache) yields an empty result.
        """
        cap = self.max_seq_len
        tasks: List[Optional[Task]] = []
        for ids in prompt_ids_list:
            if not ids or len(ids) >= cap:
                tasks.append(None)
                continue
            mt = cap - len(ids) if max_tokens is None else min(max_tokens, cap - len(ids))
            tasks.append(Task(f"batch_{uuid.uuid4().hex[:8]}", list(ids), mt, temperature, top_p, top_k,
                              frequency_penalty, rep_window))
        live_all = [t for t in tasks if t is not None]
        wave = max(1, self._task_mgr.max_batch_size)
        for i in range(0, len(live_all), wave):
            with self._step_lock:
                self._run_wave(live_all[i:i + wave])
        out: List[Any] = []
        for t in tasks:
            if t is None or t.status == TaskStatus.PENDING:
                out.append(([], []) if return_logprobs else [])
            else:
                out.append((list(t.output_ids), list(t.output_logprobs)) if return_logprobs else list(t.output_ids))
        return out

    def _run_wave(self, wave: List[Task]) -> None:
        stop_ids = self._task_mgr.tokenizer.stop_ids
        live = []
        for t in wave:
            if self._cache.task_alloc(t.task_id, t.prompt_ids):
                t.status = TaskStatus.RUNNING
                live.append(t)
        try:
            self._prefill(live)
            live = [t for t in live if not t.is_finished(stop_ids)]
            while live:
                valid = []
                for t in sorted(live, key=lambda x: x.task_id):
                    if self._cache.task_extend(t.task_id, t.next_pos):
                        valid.append(t)
                    else:
                        t.status = TaskStatus.ABORTED
                if not valid:
                    break
                self._executor.execute_decode(valid)
                live = [t for t in valid if not t.is_finished(stop_ids)]
        finally:
            for t in wave:
                self._cache.task_free(t.task_id)
