"""Tool-call extraction from generated text.

API parity with astrai/inference/api/tool_parser.py:19-344:
``BaseToolParser.feed(body, current_token_ids, delta_token_ids)`` returns
OpenAI-style deltas (``{"content": ...}`` / ``{"tool_calls": [...]}``),
``parse_complete(body)`` returns ``{"content", "tool_calls"}`` or None,
``has_tool_calls``; ``ToolParserFactory`` registers ``simple_json``
(``{"name": ..., "arguments": {...}}`` objects anywhere in the output).

This parser is incremental: :meth:`SimpleJsonToolParser.feed` scans only the
characters added since the previous call (a small JSON lexer state machine),
so streaming costs O(total length) instead of re-scanning the whole body per
token. Text that might still turn into a tool call (an open ``{`` whose
prefix can still match ``{"name":``) is held back; once it cannot, it is
released as content. Argument deltas are the raw argument text as generated,
so their concatenation is the JSON text of the arguments object (a string
``json.loads`` accepts), which is what OpenAI clients expect.
"""

from __future__ import annotations

import json
import re
import uuid
from abc import ABC, abstractmethod
from typing import Dict, List, Optional

from astrai_b200.factory import Registry

_HEAD = re.compile(r'\{\s*"name"\s*:\s*"')
_HEAD_PREFIXES = ('{', '{"', '{"n', '{"na', '{"nam', '{"name', '{"name"')


def _could_become_head(text: str) -> bool:
    """True while ``text`` (starting at '{') can still grow into ``{"name": "``."""
    if _HEAD.match(text):
        return True
    compact = re.sub(r"\s+", "", text)
    return any(compact == p for p in _HEAD_PREFIXES) or bool(re.fullmatch(r'\{"name"\s*:\s*', text.strip()))


class BaseToolParser(ABC):
    def __init__(self, tools: Optional[List[Dict]] = None, tool_choice="auto"):
        self.tools = tools or []
        self.tool_choice = tool_choice

    @abstractmethod
    def feed(self, body: str, current_token_ids: Optional[List[int]] = None,
             delta_token_ids: Optional[List[int]] = None) -> List[Dict]: ...

    @abstractmethod
    def parse_complete(self, body: str) -> Optional[Dict]: ...

    @property
    @abstractmethod
    def has_tool_calls(self) -> bool: ...


class ToolParserFactory(Registry["BaseToolParser"]):
    pass


def _scan_objects(text: str) -> List[tuple]:
    """Complete top-level ``{...}`` spans of ``text`` as (start, end)."""
    spans, depth, in_str, esc, start = [], 0, False, False, -1
    for i, c in enumerate(text):
        if in_str:
            if esc:
                esc = False
            elif c == "\\":
                esc = True
            elif c == '"':
                in_str = False
            continue
        if c == '"':
            in_str = depth > 0
        elif c == "{":
            if depth == 0:
                start = i
            depth += 1
        elif c == "}" and depth > 0:
            depth -= 1
            if depth == 0:
                spans.append((start, i + 1))
    return spans


def _as_call(obj_text: str) -> Optional[Dict]:
    try:
        obj = json.loads(obj_text)
    except json.JSONDecodeError:
        return None
    if not isinstance(obj, dict) or not isinstance(obj.get("name"), str) or not obj["name"]:
        return None
    args = obj.get("arguments", {})
    args = args if isinstance(args, str) else json.dumps(args, ensure_ascii=False)
    return {"name": obj["name"], "arguments": args}


@ToolParserFactory.register("simple_json")
class SimpleJsonToolParser(BaseToolParser):
    def __init__(self, tools=None, tool_choice="auto"):
        super().__init__(tools, tool_choice)
        self._scanned = 0          # characters of the body consumed by the lexer
        self._content_upto = 0     # characters released as content
        self._depth = 0
        self._in_str = False
        self._esc = False
        self._obj_start = -1       # start of the open top-level object
        self._calls: List[Dict] = []  # streaming state per detected call
        self._cur: Optional[Dict] = None

    @property
    def has_tool_calls(self) -> bool:
        return bool(self._calls)

    # ------------------------------------------------------------------ streaming
    def feed(self, body: str, current_token_ids=None, delta_token_ids=None) -> List[Dict]:
        out: List[Dict] = []
        i = self._scanned
        while i < len(body):
            c = body[i]
            if self._in_str:
                if self._esc:
                    self._esc = False
                elif c == "\\":
                    self._esc = True
                elif c == '"':
                    self._in_str = False
            elif c == '"' and self._depth > 0:
                self._in_str = True
            elif c == "{":
                if self._depth == 0:
                    self._obj_start = i
                self._depth += 1
            elif c == "}" and self._depth > 0:
                self._depth -= 1
                if self._depth == 0:
                    self._close_object(body, i + 1, out)
            i += 1
        self._scanned = len(body)
        if self._depth > 0 and self._obj_start >= 0:
            self._open_object(body, out)
        else:
            self._release(body, len(body), out)
        return out

    def _release(self, body: str, upto: int, out: List[Dict]) -> None:
        if upto > self._content_upto:
            text = body[self._content_upto:upto]
            self._content_upto = upto
            if text:
                out.append({"content": text})

    def _open_object(self, body: str, out: List[Dict]) -> None:
        text = body[self._obj_start:]
        if self._cur is None:
            if not _could_become_head(text):
                self._release(body, len(body), out)
                return
            m = re.match(r'\{\s*"name"\s*:\s*"((?:[^"\\]|\\.)*)"', text)
            self._release(body, self._obj_start, out)
            if not m:
                return  # still undecided: hold the text back
            self._start_call(m.group(1), out)
        self._stream_args(text, final=False, out=out)

    def _start_call(self, name: str, out: List[Dict]) -> None:
        st = {"id": f"call_{uuid.uuid4().hex[:12]}", "index": len(self._calls), "args_sent": 0}
        self._calls.append(st)
        self._cur = st
        out.append({"tool_calls": [{"index": st["index"], "id": st["id"], "type": "function",
                                    "function": {"name": name, "arguments": ""}}]})

    def _stream_args(self, text: str, final: bool, out: List[Dict]) -> None:
        m = re.search(r'"arguments"\s*:\s*', text)
        if not m or self._cur is None:
            return
        raw = text[m.end():]
        if final:  # drop the call object's closing brace
            raw = raw.rstrip()
            raw = raw[:-1].rstrip() if raw.endswith("}") else raw
        else:  # a trailing '}' may be the call object's own closing brace: hold one back
            raw = raw.rstrip()
        st = self._cur
        if len(raw) > st["args_sent"]:
            out.append({"tool_calls": [{"index": st["index"], "function": {"arguments": raw[st["args_sent"]:]}}]})
            st["args_sent"] = len(raw)

    def _close_object(self, body: str, end: int, out: List[Dict]) -> None:
        text = body[self._obj_start:end]
        if self._cur is None and _as_call(text) is not None:
            self._release(body, self._obj_start, out)
            self._start_call(json.loads(text)["name"], out)
        if self._cur is not None:
            self._stream_args(text, final=True, out=out)
            self._content_upto = end
            self._cur = None
        self._obj_start = -1

    # ------------------------------------------------------------------ whole text
    def parse_complete(self, body: str) -> Optional[Dict]:
        calls, first = [], None
        for s, e in _scan_objects(body):
            call = _as_call(body[s:e])
            if call is not None:
                first = s if first is None else first
                calls.append({"id": f"call_{uuid.uuid4().hex[:12]}", "type": "function", "function": call})
        if not calls:
            return None
        return {"content": body[:first].strip() or None, "tool_calls": calls}
