"""Generation requests and their queues.

API parity with astrai/inference/core/task.py:14-287: ``STOP`` sentinel,
``StreamDecoder`` (holds back text while the tail decodes to U+FFFD, i.e. a
multi-byte character split across byte-level BPE tokens), ``TaskStatus``,
``Task`` (prompt, sampling parameters, outputs, logprobs, stream decoding)
and the thread-safe ``TaskManager`` (waiting queue, active list, callbacks).

Position bookkeeping differs from the reference: prefill writes the prompt's
KV and samples the first token from the last prompt position, so the token
fed at decode step n is ``output_ids[-1]`` at position
``len(prompt_ids) + len(output_ids) - 1`` (no prompt token is fed twice).
"""

from __future__ import annotations

import threading
import time
import uuid
from collections import deque
from enum import Enum
from typing import Any, Callable, Deque, Dict, List, Optional

STOP = object()


class StreamDecoder:
    """Incremental detokeniser for streaming."""

    __slots__ = ("_tokenizer", "_ids", "_emitted")

    def __init__(self, tokenizer):
        self._tokenizer = tokenizer
        self._ids: List[int] = []
        self._emitted = ""

    def push(self, token_id: int) -> str:
        self._ids.append(int(token_id))
        text = self._tokenizer.decode(self._ids, skip_special_tokens=True)
        if text.endswith("�") or len(text) <= len(self._emitted):
            return ""
        new, self._emitted = text[len(self._emitted):], text
        return new

    def flush(self) -> str:
        if not self._ids:
            return ""
        text = self._tokenizer.decode(self._ids, skip_special_tokens=True)
        if len(text) <= len(self._emitted):
            return ""
        new, self._emitted = text[len(self._emitted):], text
        return new


class TaskStatus(Enum):
    PENDING = "pending"
    RUNNING = "running"
    FINISHED = "finished"
    ABORTED = "aborted"


class Task:
    def __init__(self, task_id: str, prompt_ids: List[int], max_tokens: Optional[int] = None,
                 temperature: float = 1.0, top_p: float = 1.0, top_k: int = 50, frequency_penalty: float = 0.0,
                 rep_window: int = 64):
        self.task_id = task_id
        self.prompt_ids = list(prompt_ids)
        self.max_tokens = max_tokens
        self.temperature = float(temperature)
        self.top_p = float(top_p)
        self.top_k = int(top_k)
        self.frequency_penalty = float(frequency_penalty)
        self.rep_window = int(rep_window)
        self.status = TaskStatus.PENDING
        self.output_ids: List[int] = []
        self.output_logprobs: List[float] = []
        self.input_tokens = 0
        self.output_tokens = 0
        self.arrival_time = time.time()
        self.finish_time: Optional[float] = None
        self._decoder: Optional[StreamDecoder] = None

    def decode_new_token(self, tokenizer) -> str:
        if self._decoder is None:
            self._decoder = StreamDecoder(tokenizer)
        return self._decoder.push(self.output_ids[-1])

    def flush_remaining(self, tokenizer) -> str:
        if self._decoder is None or not self.output_ids:
            return ""
        return self._decoder.flush()

    @property
    def next_pos(self) -> int:
        """Position of the token fed at the next decode step."""
        return len(self.prompt_ids) + len(self.output_ids) - 1

    def history(self) -> List[int]:
        """Frequency-penalty window: last ``rep_window`` prompt ids + all outputs."""
        return self.prompt_ids[-self.rep_window:] + self.output_ids

    def is_finished(self, stop_ids) -> bool:
        if self.max_tokens is not None and self.output_tokens >= self.max_tokens:
            return True
        return bool(self.output_ids) and self.output_ids[-1] in stop_ids


class TaskManager:
    """Waiting queue + active list + per-task stream callbacks (thread safe)."""

    def __init__(self, tokenizer, max_batch_size: int = 16, max_seq_len: int = 8192, max_prompt_len: int = 512):
        self.tokenizer = tokenizer
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.max_prompt_len = max_prompt_len
        self.waiting_queue: Deque[Task] = deque()
        self.active_tasks: List[Task] = []
        self._callbacks: Dict[str, Callable[[Any], None]] = {}
        self._event = threading.Event()
        self._lock = threading.Lock()
        self._total_tasks = 0
        self._total_tokens = 0

    def make_task(self, prompt_ids: List[int], max_tokens: Optional[int] = None, **sampling) -> Optional[Task]:
        """Truncate to ``max_prompt_len`` (keep the tail), clamp ``max_tokens``;
        None when the prompt leaves no room to generate."""
        ids = list(prompt_ids)[-self.max_prompt_len:] if self.max_prompt_len else list(prompt_ids)
        if not ids or len(ids) >= self.max_seq_len:
            return None
        room = self.max_seq_len - len(ids)
        mt = room if max_tokens is None else min(int(max_tokens), room)
        return Task(f"task_{int(time.time())}_{uuid.uuid4().hex[:8]}", ids, mt, **sampling)

    def add_task(self, prompt: str, max_tokens: Optional[int] = None, temperature: float = 1.0, top_p: float = 1.0,
                 top_k: int = 50, frequency_penalty: float = 0.0, rep_window: int = 64,
                 stream_callback: Optional[Callable[[Any], None]] = None, prompt_ids: Optional[List[int]] = None
                 ) -> str:
        ids = prompt_ids if prompt_ids is not None else self.tokenizer.encode(prompt)
        task = self.make_task(ids, max_tokens, temperature=temperature, top_p=top_p, top_k=top_k,
                              frequency_penalty=frequency_penalty, rep_window=rep_window)
        if task is None:
            if stream_callback:
                stream_callback(STOP)
            return f"task_{int(time.time())}_{uuid.uuid4().hex[:8]}"
        with self._lock:
            self.waiting_queue.append(task)
            self._total_tasks += 1
            if stream_callback:
                self._callbacks[task.task_id] = stream_callback
        self._event.set()
        return task.task_id

    def remove_task(self, task_id: str) -> List[Task]:
        with self._lock:
            removed = [t for t in self.active_tasks if t.task_id == task_id]
            self.waiting_queue = deque(t for t in self.waiting_queue if t.task_id != task_id)
            self.active_tasks = [t for t in self.active_tasks if t.task_id != task_id]
            self._callbacks.pop(task_id, None)
        return removed

    def invoke_callback(self, task_id: str, token) -> None:
        cb = self._callbacks.get(task_id)
        if cb:
            cb(token)

    def get_stats(self) -> Dict[str, Any]:
        with self._lock:
            return {"total_tasks": self._total_tasks, "total_tokens": self._total_tokens,
                    "active_tasks": len(self.active_tasks), "waiting_queue": len(self.waiting_queue)}

    def remove_finished_tasks(self, stop_ids) -> List[Task]:
        with self._lock:
            done = []
            for t in self.active_tasks:
                if t.status == TaskStatus.ABORTED:
                    done.append(t)
                elif t.is_finished(stop_ids):
                    t.status = TaskStatus.FINISHED
                    self._total_tokens += t.output_tokens
                    done.append(t)
            for t in done:
                t.finish_time = time.time()
            self.active_tasks = [t for t in self.active_tasks if t not in done]
            return done

    def pull_candidates(self, n: int) -> List[Task]:
        with self._lock:
            return [self.waiting_queue.popleft() for _ in range(min(n, len(self.waiting_queue)))]

    def activate(self, task: Task) -> None:
        task.status = TaskStatus.RUNNING
        with self._lock:
            self.active_tasks.append(task)

    def return_to_waiting(self, tasks: List[Task]) -> None:
        with self._lock:
            for t in reversed(tasks):
                self.waiting_queue.appendleft(t)

    def has_work(self) -> bool:
        with self._lock:
            return bool(self.active_tasks or self.waiting_queue)

    def wait_for_tasks(self, timeout: float = 1.0) -> None:
        with self._lock:
            if self.waiting_queue or self.active_tasks:
                return
            self._event.clear()
        self._event.wait(timeout=timeout)

    def get_active_tasks(self) -> List[Task]:
        with self._lock:
            return list(self.active_tasks)

    def get_waiting_tasks(self) -> List[Task]:
        with self._lock:
            return list(self.waiting_queue)

    def clear_queues(self) -> None:
        with self._lock:
            self.waiting_queue.clear()
            self.active_tasks.clear()
            self._callbacks.clear()

    def wake(self) -> None:
        self._event.set()
