"""Inference: paged / contiguous KV caches, fused sampling, continuous-batching
scheduler, engine facade and the OpenAI / Anthropic compatible server."""

from astrai_b200.inference.api import (AnthropicMessage, AnthropicResponseBuilder, BaseToolParser,
                                       ChatCompletionRequest, ChatMessage, FunctionDef, GenContext, MessagesRequest,
                                       OpenAIResponseBuilder, ProtocolHandler, SimpleJsonToolParser, StopChecker,
                                       ToolDef, ToolParserFactory, get_app, run_server)
from astrai_b200.inference.core import (STOP, Allocator, CacheView, ContiguousCache, ContiguousCacheView, Executor,
                                        InferenceScheduler, KVCache, PageCache, PageCacheView, PagePool, PrefixCache,
                                        Storage, StreamDecoder, Task, TaskManager, TaskStatus, TaskTable, page_hash)
from astrai_b200.inference.engine import GenerateResult, GenerationRequest, InferenceEngine
from astrai_b200.inference.sample import (BaseSamplingStrategy, DeviceRNG, FrequencyPenaltyStrategy, SamplingPipeline,
                                          TemperatureStrategy, TopKStrategy, TopPStrategy, fused_sample, sample)

__all__ = [
    "InferenceEngine", "GenerationRequest", "GenerateResult", "InferenceScheduler", "Executor", "STOP", "Task",
    "TaskManager", "TaskStatus", "StreamDecoder", "Allocator", "CacheView", "KVCache", "ContiguousCache",
    "ContiguousCacheView", "PageCache", "PageCacheView", "PagePool", "PrefixCache", "Storage", "TaskTable",
    "page_hash", "sample", "fused_sample", "DeviceRNG", "BaseSamplingStrategy", "TemperatureStrategy",
    "TopKStrategy", "TopPStrategy", "FrequencyPenaltyStrategy", "SamplingPipeline", "ProtocolHandler",
    "StopChecker", "GenContext", "BaseToolParser", "SimpleJsonToolParser", "ToolParserFactory",
    "OpenAIResponseBuilder", "AnthropicResponseBuilder", "ChatMessage", "ChatCompletionRequest", "FunctionDef",
    "ToolDef", "AnthropicMessage", "MessagesRequest", "get_app", "run_server",
]
