"""OpenAI chat-completions formatting.

Parity: astrai/inference/api/openai.py:51-277 (``OpenAIResponseBuilder``:
chat template with tools, ``chat.completion.chunk`` stream with a role
chunk first, tool-call deltas from the tool parser, ``finish_reason``
``stop`` / ``tool_calls`` / ``length``, usage). Unsupported request fields
(n, presence_penalty, logit_bias, user) are logged and ignored.
"""

from __future__ import annotations

import logging
import time
import uuid
from typing import Any, Dict, List, Optional, Tuple

from astrai_b200.inference.api.protocol import GenContext, ResponseBuilder, StopInfo, sse_event
from astrai_b200.inference.api.tool_parser import BaseToolParser, ToolParserFactory

logger = logging.getLogger(__name__)

_UNSUPPORTED = {"n": 1, "presence_penalty": 0.0, "logit_bias": None, "user": None}


def _dump(x):
    return x.model_dump() if hasattr(x, "model_dump") else x


class OpenAIResponseBuilder(ResponseBuilder):
    def prepare(self, request, engine) -> Tuple[str, GenContext, List[str]]:
        messages = []
        for m in request.messages:
            msg = {"role": m.role, "content": m.content or ""}
            if getattr(m, "tool_calls", None):
                msg["tool_calls"] = m.tool_calls
            if getattr(m, "tool_call_id", None):
                msg["tool_call_id"] = m.tool_call_id
            messages.append(msg)
        tools = [_dump(t) for t in (request.tools or [])] or None
        kwargs = {"tools": tools} if tools else {}
        prompt = engine.tokenizer.apply_chat_template(messages, tokenize=False, **kwargs)
        for name, default in _UNSUPPORTED.items():
            v = getattr(request, name, default)
            if v is not None and v != default:
                logger.warning("ChatCompletionRequest field %r=%r is not supported and is ignored", name, v)
        self._parser: Optional[BaseToolParser] = None
        choice = getattr(request, "tool_choice", "auto") or "auto"
        if tools and choice != "none":
            self._parser = ToolParserFactory.create("simple_json", tools=tools, tool_choice=choice)
        self._id = f"chatcmpl-{uuid.uuid4().hex[:24]}"
        self._model = request.model
        self._max_tokens = request.max_tokens
        self._role_sent = False
        stop = request.stop
        stops = [] if stop is None else [stop] if isinstance(stop, str) else list(stop)
        return prompt, GenContext(self._id, int(time.time()), request.model), stops

    def _chunk(self, ctx_created: int, delta: Dict[str, Any], finish: Optional[str] = None) -> str:
        return sse_event({"id": self._id, "object": "chat.completion.chunk", "created": ctx_created,
                          "model": self._model, "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]})

    def format_stream_start(self, ctx: GenContext) -> List[str]:
        self._created = ctx.created
        self._role_sent = True
        return [self._chunk(ctx.created, {"role": "assistant"})]

    def format_chunk(self, token: str, **kwargs) -> List[str]:
        created = getattr(self, "_created", int(time.time()))
        if self._parser is None:
            return [self._chunk(created, {"content": token})]
        events = []
        for d in self._parser.feed(kwargs.get("body", token), kwargs.get("current_token_ids"),
                                   kwargs.get("delta_token_ids")):
            events.append(self._chunk(created, d))
        return events

    def _finish_reason(self, ctx: GenContext, stop: StopInfo, tool_calls: bool) -> str:
        if tool_calls:
            return "tool_calls"
        if stop.matched is None and self._max_tokens and ctx.completion_tokens >= self._max_tokens:
            return "length"
        return "stop"

    def _usage(self, ctx: GenContext) -> Dict[str, int]:
        return {"prompt_tokens": ctx.prompt_tokens, "completion_tokens": ctx.completion_tokens,
                "total_tokens": ctx.prompt_tokens + ctx.completion_tokens}

    def format_stream_end(self, ctx: GenContext, stop: StopInfo) -> List[str]:
        tools = self._parser is not None and self._parser.has_tool_calls
        end = sse_event({"id": self._id, "object": "chat.completion.chunk", "created": ctx.created,
                         "model": self._model,
                         "choices": [{"index": 0, "delta": {}, "finish_reason": self._finish_reason(ctx, stop, tools)}],
                         "usage": self._usage(ctx)})
        return [end]

    def format_response(self, ctx: GenContext, content: str, stop: StopInfo) -> Dict[str, Any]:
        message: Dict[str, Any] = {"role": "assistant", "content": content}
        parsed = self._parser.parse_complete(content) if self._parser is not None else None
        if parsed:
            message = {"role": "assistant", "content": parsed["content"], "tool_calls": parsed["tool_calls"]}
        return {"id": self._id, "object": "chat.completion", "created": ctx.created, "model": self._model,
                "choices": [{"index": 0, "message": message,
                             "finish_reason": self._finish_reason(ctx, stop, bool(parsed))}],
                "usage": self._usage(ctx)}
