"""HTTP generation loop shared by the OpenAI and Anthropic endpoints.

API parity with astrai/inference/api/protocol.py:18-200 (``sse_event``,
``sse_done``, ``GenContext``, ``StopInfo``, ``StopChecker``,
``ResponseBuilder`` with five format methods, ``ProtocolHandler.handle``).

Stop sequences are handled with a hold-back window: text that could still be
the beginning of a stop sequence is not streamed until it is known not to
be one, so a matched stop sequence never leaks into the stream and the text
before it is never dropped. When a stop sequence matches, the request's task
is cancelled immediately (the async generator is closed, which removes the
task from the scheduler). ``completion_tokens`` counts generated tokens
(re-tokenised), not text pieces.
"""

from __future__ import annotations

import json
from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import Any, AsyncGenerator, Dict, List, Optional, Tuple, Union


def sse_event(data: Dict[str, Any], event: Optional[str] = None) -> str:
    head = f"event: {event}\n" if event else ""
    return f"{head}data: {json.dumps(data, ensure_ascii=False)}\n\n"


def sse_done() -> str:
    return "data: [DONE]\n\n"


@dataclass
class GenContext:
    resp_id: str
    created: int
    model: str
    prompt_tokens: int = 0
    completion_tokens: int = 0


@dataclass
class StopInfo:
    matched: Optional[str] = None
    body: str = ""
    yielded: str = ""


class StopChecker:
    """Finds the earliest stop sequence in a text and the safe-to-emit prefix."""

    def __init__(self, sequences: List[str]):
        self._seqs = [s for s in (sequences or []) if s]
        self._hold = max((len(s) for s in self._seqs), default=1) - 1

    def check(self, text: str) -> Optional[str]:
        best, where = None, len(text) + 1
        for s in self._seqs:
            i = text.find(s)
            if 0 <= i < where:
                best, where = s, i
        return best

    def cut(self, text: str) -> Tuple[Optional[str], str]:
        """-> (matched sequence or None, text that may be emitted)."""
        m = self.check(text)
        if m is not None:
            return m, text[: text.find(m)]
        if not self._seqs:
            return None, text
        # keep back the longest suffix that is a proper prefix of some stop sequence
        keep = 0
        for k in range(1, min(self._hold, len(text)) + 1):
            tail = text[-k:]
            if any(s.startswith(tail) for s in self._seqs):
                keep = k
        return None, text[: len(text) - keep]


class ResponseBuilder(ABC):
    @abstractmethod
    def prepare(self, request, engine) -> Tuple[str, GenContext, List[str]]: ...

    @abstractmethod
    def format_stream_start(self, ctx: GenContext) -> List[str]: ...

    @abstractmethod
    def format_chunk(self, token: str, **kwargs) -> List[str]: ...

    @abstractmethod
    def format_stream_end(self, ctx: GenContext, stop: StopInfo) -> List[str]: ...

    @abstractmethod
    def format_response(self, ctx: GenContext, content: str, stop: StopInfo) -> Dict[str, Any]: ...


class ProtocolHandler:
    def __init__(self, request, engine, builder: ResponseBuilder):
        self.request = request
        self.engine = engine
        self.builder = builder

    def _agen(self, prompt: str) -> AsyncGenerator[str, None]:
        r = self.request
        return self.engine.generate_async(
            prompt, max_tokens=r.max_tokens, temperature=r.temperature if r.temperature is not None else 1.0,
            top_p=r.top_p if r.top_p is not None else 1.0, top_k=r.top_k if r.top_k is not None else 50,
            frequency_penalty=getattr(r, "frequency_penalty", 0.0) or 0.0)

    def _count(self, text: str) -> int:
        return len(self.engine.tokenizer.encode(text)) if text else 0

    async def handle(self) -> Union[Any, Dict[str, Any]]:
        prompt, ctx, stops = self.builder.prepare(self.request, self.engine)
        ctx.prompt_tokens = self._count(prompt)
        agen = self._agen(prompt)
        if self.request.stream:
            from fastapi.responses import StreamingResponse

            return StreamingResponse(self._stream(agen, ctx, StopChecker(stops)), media_type="text/event-stream",
                                     headers={"Cache-Control": "no-cache", "Connection": "keep-alive"})
        return await self._collect(agen, ctx, StopChecker(stops))

    async def _stream(self, agen, ctx: GenContext, checker: StopChecker):
        for ev in self.builder.format_stream_start(ctx):
            yield ev
        body, yielded, matched = "", "", None
        try:
            async for piece in agen:
                body += piece
                matched, safe = checker.cut(body)
                if len(safe) > len(yielded):
                    new = safe[len(yielded):]
                    ids = self.engine.tokenizer.encode(safe)
                    for ev in self.builder.format_chunk(new, body=safe, current_token_ids=ids,
                                                        delta_token_ids=self.engine.tokenizer.encode(new)):
                        yield ev
                    yielded = safe
                if matched:
                    break
        finally:
            await agen.aclose()
        if not matched and len(body) > len(yielded):  # flush the held-back tail
            new = body[len(yielded):]
            for ev in self.builder.format_chunk(new, body=body):
                yield ev
            yielded = body
        ctx.completion_tokens = self._count(yielded)
        for ev in self.builder.format_stream_end(ctx, StopInfo(matched, body, yielded)):
            yield ev
        yield sse_done()

    async def _collect(self, agen, ctx: GenContext, checker: StopChecker) -> Dict[str, Any]:
        body, matched = "", None
        try:
            async for piece in agen:
                body += piece
                matched = checker.check(body)
                if matched:
                    break
        finally:
            await agen.aclose()
        content = body[: body.find(matched)] if matched else body
        ctx.completion_tokens = self._count(content)
        return self.builder.format_response(ctx, content, StopInfo(matched, body, content))
