"""Generation requests and the queues the scheduler serves them from.

Public names kept from the reference (astrai/inference/core/task.py:14-287): ``STOP`` (the
end-of-stream sentinel handed to stream callbacks), ``StreamDecoder``, ``TaskStatus``, ``Task``
and ``TaskManager``.

* :class:`StreamDecoder` turns generated ids into text incrementally with a two-offset window
  (the incremental detokenisation scheme used by several open serving engines): each push
  decodes only ``ids[prefix:]`` and compares it with ``ids[prefix:read]``, so the cost per token
  does not grow with the output length. Text is held back while it ends in U+FFFD, i.e. while a
  multi-byte character is split across byte-level BPE tokens. Because the window starts one
  chunk before the new tokens, tokenizers that strip a leading space at the start of a decode
  still produce the space of a new word.
* :class:`Task` is a dataclass of the prompt, the sampling parameters, the outputs and the
  stream callback. Position bookkeeping: prefill writes the prompt's KV and samples the first
  token from the last prompt position, so the token fed at a decode step is ``output_ids[-1]``
  at position ``len(prompt_ids) + len(output_ids) - 1`` (no prompt token is fed twice).
* :class:`TaskManager` keeps a waiting deque and an id-ordered dict of active tasks under one
  condition variable; the scheduler thread sleeps on it when there is no work.
"""

from __future__ import annotations

import itertools
import threading
import time
from collections import OrderedDict, deque
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Callable, Deque, Dict, List, Optional

STOP = object()

Callback = Callable[[Any], None]
_ids = itertools.count()


def _new_id(kind: str = "task") -> str:
    return f"{kind}_{next(_ids)}_{time.monotonic_ns() & 0xFFFFFF:06x}"


class StreamDecoder:
    """Incremental detokeniser: ``push(id)`` returns the newly completed text (maybe empty),
    ``flush()`` whatever is still held back at the end."""

    __slots__ = ("_tok", "_ids", "_prefix", "_read")

    def __init__(self, tokenizer):
        self._tok = tokenizer
        self._ids: List[int] = []
        self._prefix = 0  # window start (one emitted chunk before the unread tokens)
        self._read = 0  # ids before this index are emitted

    def _text(self, lo: int, hi: Optional[int] = None) -> str:
        return self._tok.decode(self._ids[lo:hi], skip_special_tokens=True)

    def _advance(self, final: bool) -> str:
        seen = self._text(self._prefix, self._read)
        now = self._text(self._prefix)
        if len(now) <= len(seen) or (now.endswith("�") and not final):
            return ""
        self._prefix, self._read = self._read, len(self._ids)
        return now[len(seen):]

    def push(self, token_id: int) -> str:
        self._ids.append(int(token_id))
        return self._advance(final=False)

    def flush(self) -> str:
        return self._advance(final=True) if self._read < len(self._ids) else ""


class TaskStatus(Enum):
    PENDING = "pending"
    RUNNING = "running"
    FINISHED = "finished"
    ABORTED = "aborted"


@dataclass(eq=False)
class Task:
    task_id: str
    prompt_ids: List[int]
    max_tokens: Optional[int] = None
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 50
    frequency_penalty: float = 0.0
    rep_window: int = 64
    callback: Optional[Callback] = None
    status: TaskStatus = TaskStatus.PENDING
    output_ids: List[int] = field(default_factory=list)
    output_logprobs: List[float] = field(default_factory=list)
    input_tokens: int = 0
    output_tokens: int = 0
    arrival_time: float = field(default_factory=time.time)
    finish_time: Optional[float] = None
    _detok: Optional[StreamDecoder] = field(default=None, repr=False)

    def __post_init__(self):
        self.prompt_ids = list(self.prompt_ids)
        self.temperature, self.top_p = float(self.temperature), float(self.top_p)
        self.top_k, self.rep_window = int(self.top_k), int(self.rep_window)
        self.frequency_penalty = float(self.frequency_penalty)

    # ------------------------------------------------------------------ streaming text
    def decode_new_token(self, tokenizer) -> str:
        """Text completed by the newest output id."""
        if self._detok is None:
            self._detok = StreamDecoder(tokenizer)
        return self._detok.push(self.output_ids[-1])

    def flush_remaining(self, tokenizer) -> str:
        """Text still held back when the task ends."""
        return self._detok.flush() if self._detok is not None else ""

    # ------------------------------------------------------------------ bookkeeping
    @property
    def next_pos(self) -> int:
        """Position of the token fed at the next decode step."""
        return len(self.prompt_ids) + len(self.output_ids) - 1

    def history(self) -> List[int]:
        """Ids the frequency penalty counts: the last ``rep_window`` prompt ids and every output."""
        return self.prompt_ids[-self.rep_window:] + self.output_ids

    def is_finished(self, stop_ids) -> bool:
        if self.max_tokens is not None and self.output_tokens >= self.max_tokens:
            return True
        return bool(self.output_ids) and self.output_ids[-1] in stop_ids

    def notify(self, piece: Any) -> None:
        if self.callback is not None:
            self.callback(piece)


class TaskManager:
    """Thread-safe waiting queue + active set of one scheduler."""

    def __init__(self, tokenizer, max_batch_size: int = 16, max_seq_len: int = 8192, max_prompt_len: int = 512):
        self.tokenizer = tokenizer
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.max_prompt_len = max_prompt_len
        self._cv = threading.Condition()
        self._waiting: Deque[Task] = deque()
        self._active: "OrderedDict[str, Task]" = OrderedDict()
        self._submitted = 0
        self._generated = 0

    # ------------------------------------------------------------------ admission
    def make_task(self, prompt_ids: List[int], max_tokens: Optional[int] = None, **sampling) -> Optional[Task]:
        """A task for ``prompt_ids`` cut to its last ``max_prompt_len`` ids, with ``max_tokens``
        clamped to the room left in ``max_seq_len``; None when no room is left."""
        ids = list(prompt_ids)
        if self.max_prompt_len:
            ids = ids[-self.max_prompt_len:]
        room = self.max_seq_len - len(ids)
        if not ids or room <= 0:
            return None
        budget = room if max_tokens is None else min(int(max_tokens), room)
        return Task(_new_id(), ids, budget, **sampling)

    def add_task(self, prompt: str, max_tokens: Optional[int] = None, temperature: float = 1.0, top_p: float = 1.0,
                 top_k: int = 50, frequency_penalty: float = 0.0, rep_window: int = 64,
                 stream_callback: Optional[Callback] = None, prompt_ids: Optional[List[int]] = None) -> str:
        """Queue a request; returns its id. A prompt that leaves no room to generate is answered
        with ``STOP`` at once (its id is still returned, and refers to nothing)."""
        ids = self.tokenizer.encode(prompt) if prompt_ids is None else prompt_ids
        task = self.make_task(ids, max_tokens, temperature=temperature, top_p=top_p, top_k=top_k,
                              frequency_penalty=frequency_penalty, rep_window=rep_window)
        if task is None:
            if stream_callback is not None:
                stream_callback(STOP)
            return _new_id("rejected")
        task.callback = stream_callback
        with self._cv:
            self._waiting.append(task)
            self._submitted += 1
            self._cv.notify_all()
        return task.task_id

    def remove_task(self, task_id: str) -> List[Task]:
        """Drop a task wherever it is; returns it if it was active (its cache must be freed)."""
        with self._cv:
            gone = self._active.pop(task_id, None)
            self._waiting = deque(t for t in self._waiting if t.task_id != task_id)
        if gone is not None:
            gone.callback = None
            return [gone]
        return []

    def invoke_callback(self, task_id: str, token) -> None:
        with self._cv:
            task = self._active.get(task_id) or next((t for t in self._waiting if t.task_id == task_id), None)
        if task is not None:
            task.notify(token)

    # ------------------------------------------------------------------ scheduler side
    def pull_candidates(self, n: int) -> List[Task]:
        with self._cv:
            return [self._waiting.popleft() for _ in range(min(n, len(self._waiting)))]

    def return_to_waiting(self, tasks: List[Task]) -> None:
        with self._cv:
            self._waiting.extendleft(reversed(tasks))

    def activate(self, task: Task) -> None:
        task.status = TaskStatus.RUNNING
        with self._cv:
            self._active[task.task_id] = task

    def remove_finished_tasks(self, stop_ids) -> List[Task]:
        """Retire aborted tasks and tasks that hit a stop id or their token budget."""
        now = time.time()
        with self._cv:
            done = [t for t in self._active.values() if t.status == TaskStatus.ABORTED or t.is_finished(stop_ids)]
            for t in done:
                del self._active[t.task_id]
                t.finish_time = now
                if t.status != TaskStatus.ABORTED:
                    t.status = TaskStatus.FINISHED
                    self._generated += t.output_tokens
        return done

    def has_work(self) -> bool:
        with self._cv:
            return bool(self._active or self._waiting)

    def wait_for_tasks(self, timeout: float = 1.0) -> None:
        """Sleep until a task arrives, :meth:`wake` is called, or ``timeout`` passes."""
        with self._cv:
            if not (self._active or self._waiting):
                self._cv.wait(timeout)

    def wake(self) -> None:
        with self._cv:
            self._cv.notify_all()

    def get_active_tasks(self) -> List[Task]:
        with self._cv:
            return list(self._active.values())

    def get_waiting_tasks(self) -> List[Task]:
        with self._cv:
            return list(self._waiting)

    def clear_queues(self) -> None:
        with self._cv:
            self._waiting.clear()
            self._active.clear()

    def get_stats(self) -> Dict[str, Any]:
        with self._cv:
            return {"total_tasks": self._submitted, "total_tokens": self._generated,
                    "active_tasks": len(self._active), "waiting_queue": len(self._waiting)}

    # the scheduler and tests read these two as lists
    @property
    def active_tasks(self) -> List[Task]:
        return self.get_active_tasks()

    @property
    def waiting_queue(self) -> List[Task]:
        return self.get_waiting_tasks()
