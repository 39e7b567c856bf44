"""Anthropic Messages formatting.

Parity: astrai/inference/api/anthropic.py:28-142 (system prompt + text
blocks through the chat template; ``message_start``,
``content_block_start``, ``content_block_delta`` (text_delta),
``content_block_stop``, ``message_delta`` with ``stop_reason``
``end_turn`` / ``stop_sequence`` / ``max_tokens``, ``message_stop``).
The generation loop already withholds stop sequences, so no trimming
happens here.
"""

from __future__ import annotations

import time
import uuid
from typing import Any, Dict, List, Tuple

from astrai_b200.inference.api.protocol import GenContext, ResponseBuilder, StopInfo, sse_event


def _text_of(content) -> str:
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        return "".join(b.get("text", "") for b in content if isinstance(b, dict) and b.get("type") == "text")
    return ""


class AnthropicResponseBuilder(ResponseBuilder):
    def prepare(self, request, engine) -> Tuple[str, GenContext, List[str]]:
        messages = []
        if getattr(request, "system", None):
            messages.append({"role": "system", "content": request.system})
        for m in request.messages:
            text = _text_of(m.content)
            if text:
                messages.append({"role": m.role, "content": text})
        prompt = engine.tokenizer.apply_chat_template(messages, tokenize=False)
        self._max_tokens = request.max_tokens
        ctx = GenContext(f"msg_{uuid.uuid4().hex[:24]}", int(time.time()), request.model)
        return prompt, ctx, list(getattr(request, "stop_sequences", None) or [])

    def _reason(self, ctx: GenContext, stop: StopInfo) -> str:
        if stop.matched:
            return "stop_sequence"
        if self._max_tokens and ctx.completion_tokens >= self._max_tokens:
            return "max_tokens"
        return "end_turn"

    def format_stream_start(self, ctx: GenContext) -> List[str]:
        msg = {"id": ctx.resp_id, "type": "message", "role": "assistant", "model": ctx.model, "content": [],
               "stop_reason": None, "stop_sequence": None, "usage": {"input_tokens": ctx.prompt_tokens,
                                                                      "output_tokens": 0}}
        return [sse_event({"type": "message_start", "message": msg}, event="message_start"),
                sse_event({"type": "content_block_start", "index": 0, "content_block": {"type": "text", "text": ""}},
                          event="content_block_start")]

    def format_chunk(self, token: str, **kwargs) -> List[str]:
        return [sse_event({"type": "content_block_delta", "index": 0, "delta": {"type": "text_delta", "text": token}},
                          event="content_block_delta")]

    def format_stream_end(self, ctx: GenContext, stop: StopInfo) -> List[str]:
        return [sse_event({"type": "content_block_stop", "index": 0}, event="content_block_stop"),
                sse_event({"type": "message_delta",
                           "delta": {"stop_reason": self._reason(ctx, stop), "stop_sequence": stop.matched},
                           "usage": {"output_tokens": ctx.completion_tokens}}, event="message_delta"),
                sse_event({"type": "message_stop"}, event="message_stop")]

    def format_response(self, ctx: GenContext, content: str, stop: StopInfo) -> Dict[str, Any]:
        return {"id": ctx.resp_id, "type": "message", "role": "assistant", "model": ctx.model,
                "content": [{"type": "text", "text": content}], "stop_reason": self._reason(ctx, stop),
                "stop_sequence": stop.matched,
                "usage": {"input_tokens": ctx.prompt_tokens, "output_tokens": ctx.completion_tokens}}
