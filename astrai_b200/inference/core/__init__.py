"""Inference core: KV caches, tasks, executor, continuous-batching scheduler."""

from astrai_b200.inference.core.cache import (
    Allocator,
    CacheView,
    ContiguousCache,
    ContiguousCacheView,
    KVCache,
    PageCache,
    PageCacheView,
    PagePool,
    PrefixCache,
    Storage,
    TaskTable,
    page_hash,
)
from astrai_b200.inference.core.executor import Executor
from astrai_b200.inference.core.scheduler import InferenceScheduler
from astrai_b200.inference.core.task import STOP, StreamDecoder, Task, TaskManager, TaskStatus

__all__ = ["Allocator", "CacheView", "ContiguousCache", "ContiguousCacheView", "Executor", "InferenceScheduler",
           "KVCache", "PageCache", "PageCacheView", "PagePool", "PrefixCache", "STOP", "Storage", "StreamDecoder",
           "Task", "TaskManager", "TaskStatus", "TaskTable", "page_hash"]
