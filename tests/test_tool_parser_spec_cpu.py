"""Tool-call parser behaviour, case by case: whole-text parsing (parse_complete), streaming deltas (feed),
call ids, the factory, and token ids. Each case states the behaviour a client of the OpenAI-compatible
server relies on; the cases follow the reference project's parser suite as a specification
(tests/inference/test_tool_parser.py there), written against this parser's public API."""

import json

import pytest

from astrai_b200.inference.api.tool_parser import BaseToolParser, SimpleJsonToolParser, ToolParserFactory


def parser(**kw):
    return ToolParserFactory.create("simple_json", **kw)


def complete(text):
    return parser().parse_complete(text)


def stream(text, step=1):
    """Feed growing prefixes (``step`` characters at a time); return (parser, deltas)."""
    p, deltas = parser(), []
    for end in list(range(step, len(text), step)) + [len(text)]:
        deltas += p.feed(text[:end])
    return p, deltas


def merged(deltas):
    content = "".join(d.get("content", "") for d in deltas)
    calls = {}
    for d in deltas:
        for tc in d.get("tool_calls", []):
            slot = calls.setdefault(tc["index"], {"id": None, "name": "", "arguments": ""})
            slot["id"] = tc.get("id") or slot["id"]
            fn = tc.get("function", {})
            slot["name"] += fn.get("name") or ""
            slot["arguments"] += fn.get("arguments") or ""
    return content, [calls[i] for i in sorted(calls)]


def args_of(call):
    return json.loads(call["function"]["arguments"])


# ---------------------------------------------------------------------------------------- parse_complete
def test_complete_single_call():
    r = complete('{"name": "get_weather", "arguments": {"city": "Beijing"}}')
    assert [c["function"]["name"] for c in r["tool_calls"]] == ["get_weather"]
    assert args_of(r["tool_calls"][0]) == {"city": "Beijing"}


def test_complete_text_before_call_is_content():
    r = complete('Let me check. {"name": "f", "arguments": {}}')
    assert r["content"] == "Let me check." and r["tool_calls"][0]["function"]["name"] == "f"


def test_complete_two_adjacent_calls():
    r = complete('{"name": "f1", "arguments": {"a": 1}}{"name": "f2", "arguments": {"b": 2}}')
    assert [c["function"]["name"] for c in r["tool_calls"]] == ["f1", "f2"]
    assert args_of(r["tool_calls"][1]) == {"b": 2}


def test_complete_calls_separated_by_text():
    r = complete('A {"name": "x", "arguments": {}} B {"name": "y", "arguments": {"k": 1}}')
    assert [c["function"]["name"] for c in r["tool_calls"]] == ["x", "y"] and r["content"] == "A"


def test_complete_without_call_is_none():
    assert complete("The weather is nice today.") is None


def test_complete_plain_json_object_is_not_a_call():
    assert complete('{"city": "Paris", "temp": 21}') is None


def test_complete_skips_non_call_json_before_a_call():
    r = complete('{"x": 1} then {"name": "f", "arguments": {"y": 2}}')
    assert len(r["tool_calls"]) == 1 and args_of(r["tool_calls"][0]) == {"y": 2}


def test_complete_missing_arguments_means_empty_object():
    r = complete('{"name": "ping"}')
    assert r["tool_calls"][0]["function"]["name"] == "ping" and args_of(r["tool_calls"][0]) == {}


def test_complete_deeply_nested_arguments():
    nested = {"a": {"b": {"c": {"d": {"e": [1, {"f": "g"}]}}}}}
    r = complete(json.dumps({"name": "deep", "arguments": nested}))
    assert args_of(r["tool_calls"][0]) == nested


def test_complete_booleans_and_null():
    r = complete('{"name": "f", "arguments": {"t": true, "f": false, "n": null}}')
    assert args_of(r["tool_calls"][0]) == {"t": True, "f": False, "n": None}


def test_complete_array_argument():
    r = complete('{"name": "f", "arguments": {"xs": [1, 2, 3]}}')
    assert args_of(r["tool_calls"][0]) == {"xs": [1, 2, 3]}


def test_complete_array_of_objects():
    r = complete('{"name": "f", "arguments": {"rows": [{"id": 1}, {"id": 2, "tags": ["a"]}]}}')
    assert args_of(r["tool_calls"][0])["rows"][1]["tags"] == ["a"]


def test_complete_arguments_given_as_string_pass_through():
    r = complete('{"name": "f", "arguments": "{\\"q\\": 1}"}')
    assert r["tool_calls"][0]["function"]["arguments"] == '{"q": 1}'


def test_complete_unicode_arguments_are_kept():
    r = complete('{"name": "geo", "arguments": {"city": "北京", "note": "café ✓"}}')
    assert args_of(r["tool_calls"][0]) == {"city": "北京", "note": "café ✓"}


def test_complete_escaped_quotes_in_arguments():
    r = complete(r'{"name": "say", "arguments": {"text": "he said \"hi\""}}')
    assert args_of(r["tool_calls"][0]) == {"text": 'he said "hi"'}


def test_complete_braces_inside_strings_do_not_end_the_call():
    r = complete('{"name": "code", "arguments": {"src": "function() { return {}; }"}}')
    assert args_of(r["tool_calls"][0]) == {"src": "function() { return {}; }"}


def test_complete_many_properties():
    props = {f"k{i}": i for i in range(40)}
    r = complete(json.dumps({"name": "wide", "arguments": props}))
    assert args_of(r["tool_calls"][0]) == props


def test_complete_empty_arguments_object():
    r = complete('{"name": "noop", "arguments": {}}')
    assert args_of(r["tool_calls"][0]) == {}


def test_complete_whitespace_inside_call_object():
    r = complete('{ \n "name" :  "spaced" ,\n "arguments" : { "k" : "v" } \n}')
    assert r["tool_calls"][0]["function"]["name"] == "spaced" and args_of(r["tool_calls"][0]) == {"k": "v"}


def test_complete_unterminated_call_is_not_a_call():
    assert complete('{"name": "f", "arguments": {"a": 1') is None


def test_complete_content_none_for_pure_call():
    assert complete('{"name": "f", "arguments": {}}')["content"] is None


def test_complete_ids_are_unique_and_prefixed():
    r = complete('{"name": "a", "arguments": {}}{"name": "b", "arguments": {}}')
    ids = [c["id"] for c in r["tool_calls"]]
    assert len(set(ids)) == 2 and all(i.startswith("call_") for i in ids)
    assert all(c["type"] == "function" for c in r["tool_calls"])


def test_complete_real_world_search_call():
    text = ('I will search for that.\n{"name": "web_search", "arguments": {"query": "B200 HBM3e bandwidth", '
            '"top_k": 5, "filters": {"site": ["nvidia.com"], "recent": true}}}')
    r = complete(text)
    a = args_of(r["tool_calls"][0])
    assert r["content"] == "I will search for that." and a["filters"]["site"] == ["nvidia.com"] and a["top_k"] == 5


def test_complete_empty_name_is_not_a_call():
    assert complete('{"name": "", "arguments": {}}') is None


def test_complete_non_string_name_is_not_a_call():
    assert complete('{"name": 7, "arguments": {}}') is None


# ---------------------------------------------------------------------------------------- feed
def test_feed_plain_text_streams_as_content():
    p, deltas = stream("hello there", step=3)
    content, calls = merged(deltas)
    assert content == "hello there" and calls == [] and not p.has_tool_calls


def test_feed_returns_only_new_text():
    p = parser()
    assert merged(p.feed("abc"))[0] == "abc"
    assert merged(p.feed("abcdef"))[0] == "def"


def test_feed_same_body_twice_emits_nothing():
    p = parser()
    p.feed("abc")
    assert p.feed("abc") == []


def test_feed_name_arrives_before_the_arguments():
    p = parser()
    first = p.feed('{"name": "get_time", "arguments": ')
    content, calls = merged(first)
    assert calls and calls[0]["name"] == "get_time" and calls[0]["arguments"] == ""
    assert content == ""


def test_feed_arguments_stream_in_pieces():
    text = '{"name": "f", "arguments": {"city": "Paris", "days": 3}}'
    _, deltas = stream(text, step=4)
    arg_deltas = [tc["function"]["arguments"] for d in deltas for tc in d.get("tool_calls", [])
                  if tc.get("function", {}).get("arguments")]
    assert len(arg_deltas) > 1
    assert json.loads("".join(arg_deltas)) == {"city": "Paris", "days": 3}


def test_feed_text_before_call_is_released_before_the_call():
    _, deltas = stream('Sure! {"name": "f", "arguments": {}}', step=2)
    kinds = ["content" if "content" in d else "call" for d in deltas]
    assert kinds[0] == "content" and "call" in kinds
    assert merged(deltas)[0] == "Sure! "


def test_has_tool_calls_false_before_any_call():
    assert parser().has_tool_calls is False


def test_has_tool_calls_true_once_a_call_starts():
    p = parser()
    p.feed('{"name": "f", "arg')
    assert p.has_tool_calls is True


def test_feed_two_calls_get_indices_0_and_1():
    _, deltas = stream('{"name": "a", "arguments": {"x": 1}}{"name": "b", "arguments": {"y": 2}}', step=5)
    _, calls = merged(deltas)
    assert [c["name"] for c in calls] == ["a", "b"]
    assert [json.loads(c["arguments"]) for c in calls] == [{"x": 1}, {"y": 2}]


def test_feed_constructor_accepts_tools():
    tools = [{"type": "function", "function": {"name": "f", "parameters": {}}}]
    p = SimpleJsonToolParser(tools=tools)
    assert p.tools == tools
    assert merged(p.feed('{"name": "f", "arguments": {}}'))[1][0]["name"] == "f"


def test_feed_text_after_a_call_is_content():
    _, deltas = stream('{"name": "f", "arguments": {}} and more', step=3)
    content, calls = merged(deltas)
    assert len(calls) == 1 and content.strip() == "and more"


def test_feed_token_by_token_matches_complete_parse():
    text = '{"name": "lookup", "arguments": {"id": 42, "fields": ["a", "b"]}}'
    _, deltas = stream(text, step=1)
    _, calls = merged(deltas)
    ref = complete(text)["tool_calls"][0]
    assert calls[0]["name"] == ref["function"]["name"]
    assert json.loads(calls[0]["arguments"]) == args_of(ref)


def test_feed_token_by_token_text_then_call():
    _, deltas = stream('Checking now. {"name": "check", "arguments": {"ok": true}}', step=1)
    content, calls = merged(deltas)
    assert content == "Checking now. " and json.loads(calls[0]["arguments"]) == {"ok": True}


def test_feed_nested_arguments_token_by_token():
    args = {"a": {"b": [1, {"c": "}{"}]}}
    _, deltas = stream(json.dumps({"name": "n", "arguments": args}), step=1)
    assert json.loads(merged(deltas)[1][0]["arguments"]) == args


def test_feed_unicode_arguments_token_by_token():
    args = {"q": "东京 → Kyōto"}
    _, deltas = stream(json.dumps({"name": "route", "arguments": args}, ensure_ascii=False), step=1)
    assert json.loads(merged(deltas)[1][0]["arguments"]) == args


def test_feed_array_arguments_token_by_token():
    _, deltas = stream('{"name": "sum", "arguments": {"xs": [1, 2, 3, 4]}}', step=1)
    assert json.loads(merged(deltas)[1][0]["arguments"]) == {"xs": [1, 2, 3, 4]}


def test_feed_empty_arguments_stream():
    _, deltas = stream('{"name": "noop", "arguments": {}}', step=1)
    assert json.loads(merged(deltas)[1][0]["arguments"]) == {}


def test_feed_argument_deltas_never_repeat_text():
    text = '{"name": "f", "arguments": {"long": "' + "x" * 50 + '"}}'
    _, deltas = stream(text, step=7)
    pieces = [tc["function"]["arguments"] for d in deltas for tc in d.get("tool_calls", [])
              if tc.get("function", {}).get("arguments")]
    assert "".join(pieces) == '{"long": "' + "x" * 50 + '"}'


def test_feed_each_call_has_its_own_id():
    _, deltas = stream('{"name": "a", "arguments": {}}{"name": "b", "arguments": {}}', step=4)
    ids = [tc["id"] for d in deltas for tc in d.get("tool_calls", []) if "id" in tc]
    assert len(ids) == 2 and len(set(ids)) == 2


def test_feed_non_call_json_is_released_as_content():
    _, deltas = stream('result: {"x": 1} ok', step=2)
    content, calls = merged(deltas)
    assert calls == [] and content == 'result: {"x": 1} ok'


def test_feed_holds_back_a_possible_call_start():
    p = parser()
    assert merged(p.feed('text {"na'))[0] == "text "


def test_feed_then_parse_complete_on_the_same_instance():
    text = 'x {"name": "f", "arguments": {"a": [1]}}'
    p = parser()
    for end in range(1, len(text) + 1):
        p.feed(text[:end])
    r = p.parse_complete(text)
    assert r["content"] == "x" and args_of(r["tool_calls"][0]) == {"a": [1]}


# ---------------------------------------------------------------------------------------- factory / ids
def test_factory_lists_simple_json():
    assert "simple_json" in ToolParserFactory.list_registered()


def test_factory_creates_the_registered_class():
    assert isinstance(ToolParserFactory.create("simple_json"), SimpleJsonToolParser)


def test_factory_passes_tools_through():
    tools = [{"type": "function", "function": {"name": "x"}}]
    assert ToolParserFactory.create("simple_json", tools=tools).tools == tools


def test_factory_drops_unknown_keyword_arguments():
    p = ToolParserFactory.create("simple_json", tools=None, not_a_parameter=3)
    assert isinstance(p, SimpleJsonToolParser) and p.tools == []


def test_factory_registers_a_custom_parser():
    @ToolParserFactory.register("always_none_test")
    class NoCalls(BaseToolParser):
        def feed(self, body, current_token_ids=None, delta_token_ids=None):
            return [{"content": body}]

        def parse_complete(self, body):
            return None

        @property
        def has_tool_calls(self):
            return False

    p = ToolParserFactory.create("always_none_test")
    assert isinstance(p, NoCalls) and p.parse_complete('{"name": "f"}') is None


def test_token_ids_are_accepted_and_do_not_change_results():
    text = '{"name": "f", "arguments": {"a": 1}}'
    p1, p2 = parser(), parser()
    d1 = p1.feed(text)
    d2 = p2.feed(text, current_token_ids=list(range(30)), delta_token_ids=[29])
    strip = lambda ds: [{k: v for k, v in d.items() if k != "tool_calls"} for d in ds]  # noqa: E731
    assert merged(d1)[1][0]["name"] == merged(d2)[1][0]["name"] and strip(d1) == strip(d2)
    assert merged(d1)[1][0]["arguments"] == merged(d2)[1][0]["arguments"]


def test_base_parser_is_abstract():
    with pytest.raises(TypeError):
        BaseToolParser()
