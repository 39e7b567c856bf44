"""Streaming tool-call parser: every split of the output into chunks yields the same calls and content as
parsing the whole text; arguments stream as the raw JSON text of the arguments object."""

import json
import random

import pytest

CASES = [
    ("plain text without calls", 0),
    ('{"name": "get_weather", "arguments": {"city": "Paris", "unit": "C"}}', 1),
    ('Sure. {"name": "add", "arguments": {"a": 1, "b": [1, 2, {"c": "}"}]}} done', 1),
    ('{"name":"a","arguments":{}}{"name":"b","arguments":{"x":"{\\"y\\"}"}}', 2),
    ('set {"x": 1} is not a call', 0),
    ('{"nam', 0),
    ('prefix { "name" : "spaced", "arguments" : {"k": "v"} } suffix', 1),
    ('{"name": "unicode", "arguments": {"s": "héllo ✓ 你好"}}', 1),
]


def _parser():
    from astrai_b200.inference.api.tool_parser import ToolParserFactory

    return ToolParserFactory.create("simple_json")


def _stream(text, cuts):
    p = _parser()
    body, deltas = "", []
    prev = 0
    for c in list(cuts) + [len(text)]:
        body = text[:c]
        if c > prev:
            deltas += p.feed(body)
        prev = c
    return p, deltas


def _collect(deltas):
    content = "".join(d.get("content", "") for d in deltas)
    calls = {}
    for d in deltas:
        for tc in d.get("tool_calls", []):
            slot = calls.setdefault(tc["index"], {"name": "", "arguments": ""})
            fn = tc.get("function", {})
            slot["name"] += fn.get("name") or ""
            slot["arguments"] += fn.get("arguments") or ""
    return content, [calls[i] for i in sorted(calls)]


@pytest.mark.parametrize("text,n_calls", CASES)
def test_every_chunking_matches_complete_parse(text, n_calls):
    complete = _parser().parse_complete(text)
    got_calls = complete["tool_calls"] if complete else []
    assert len(got_calls) == n_calls
    rng = random.Random(hash(text) & 0xffff)
    for trial in range(25):
        k = rng.randint(0, min(len(text), 12))
        cuts = sorted(rng.sample(range(1, len(text) + 1), k)) if text else []
        if trial == 0:
            cuts = list(range(1, len(text)))  # one character at a time
        p, deltas = _stream(text, cuts)
        content, calls = _collect(deltas)
        assert len(calls) == n_calls, (cuts, deltas)
        for c, ref in zip(calls, got_calls):
            assert c["name"] == ref["function"]["name"]
            assert json.loads(c["arguments"]) == json.loads(ref["function"]["arguments"])
        assert p.has_tool_calls == (n_calls > 0)
        if n_calls == 0:
            # text that is not a call is eventually released as content (possibly held until the end)
            assert text.startswith(content)


def test_content_around_calls_is_preserved():
    text = 'Before {"name": "f", "arguments": {"a": 1}} after'
    _, deltas = _stream(text, list(range(1, len(text))))
    content, calls = _collect(deltas)
    assert content.startswith("Before") and calls[0]["name"] == "f"


def test_unterminated_call_streams_its_start_but_is_not_complete():
    text = '{"name": "unterminated", "arguments": {"a": 1'
    _, deltas = _stream(text, list(range(1, len(text))))
    _, calls = _collect(deltas)
    # streaming cannot know the object never closes: the name and argument text already went out
    assert calls and calls[0]["name"] == "unterminated" and calls[0]["arguments"] == '{"a": 1'
    assert _parser().parse_complete(text) is None
