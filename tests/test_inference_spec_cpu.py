"""Inference layers on CPU: page allocator / prefix cache / task table, tasks and the task manager,
the engine's per-call event FIFO, the incremental detokeniser, the sampling strategies, stop-sequence
handling, the OpenAI / Anthropic response builders and the HTTP server (test client, stub engine),
and scheduler thread safety. Behaviour the reference's inference suite specifies
(tests/inference/*.py there), written against this framework's public API."""

import asyncio
import json
import threading

import pytest
import torch

from astrai_b200.inference import (STOP, Allocator, PagePool, PrefixCache, StreamDecoder, Task, TaskManager,
                                   TaskStatus, TaskTable, page_hash)
from astrai_b200.inference.api.protocol import GenContext, StopChecker, StopInfo
from astrai_b200.inference.engine import GenerateResult, GenerationRequest
from astrai_b200.inference.sample import (FrequencyPenaltyStrategy, SamplingPipeline, TemperatureStrategy,
                                          TopKStrategy, TopPStrategy, sample)


# ---------------------------------------------------------------------------------------- page hashing / pools
def test_page_hash_is_deterministic():
    ids = list(range(16))
    assert page_hash(ids, 1, 8) == page_hash(list(ids), 1, 8)


def test_page_hash_differs_for_different_pages():
    assert page_hash([1, 2, 3, 4], 0, 4) != page_hash([1, 2, 3, 5], 0, 4)


def test_allocator_gives_the_lowest_free_page_first():
    a = Allocator(4)
    assert [a.alloc() for _ in range(4)] == [0, 1, 2, 3]
    a.free(2)
    a.free(0)
    assert a.alloc() == 0 and a.alloc() == 2


def test_allocator_reports_exhaustion():
    a = Allocator(1)
    assert a.alloc() == 0 and a.alloc() == -1 and a.num_free == 0


def test_allocator_inc_ref_keeps_a_page_alive():
    a = Allocator(2)
    p = a.alloc()
    a.inc_ref(p)
    a.free(p)
    assert a.ref_count(p) == 1 and a.num_free == 1


def test_cached_free_page_is_reused_by_hash_before_eviction():
    pool = PagePool(Allocator(2), PrefixCache(4))
    ids = [1, 2, 3, 4]
    p = pool.alloc()
    pool.record(p, ids, 0)
    pool.free(p)  # hashed: kept in the LRU, not freed
    assert pool.lookup(ids) == [p]
    pool.inc_ref(p)
    assert pool.allocator.ref_count(p) == 1


def test_cached_pages_are_evicted_when_the_pool_runs_dry():
    pool = PagePool(Allocator(1), PrefixCache(2))
    p = pool.alloc()
    pool.record(p, [7, 8], 0)
    pool.free(p)
    q = pool.alloc()  # no free page: the cached one is evicted and its hash forgotten
    assert q == p and pool.lookup([7, 8]) == []


def test_prefix_lookup_stops_at_the_first_miss():
    pc = PrefixCache(2)
    ids = [1, 2, 3, 4, 5, 6]
    pc.record(10, ids, 0)
    pc.record(12, ids, 2)  # page 1 missing
    assert pc.lookup(ids) == [10]


def test_prefix_lookup_ignores_a_partial_last_page():
    pc = PrefixCache(4)
    pc.record(3, [1, 2, 3, 4, 5, 6, 7, 8], 0)
    assert pc.lookup([1, 2, 3, 4, 5]) == [3] and pc.lookup([1, 2, 3]) == []


def test_prefix_evict_forgets_the_page():
    pc = PrefixCache(2)
    pc.record(5, [1, 2], 0)
    assert pc.has_page(5)
    pc.evict(5)
    assert not pc.has_page(5) and pc.lookup([1, 2]) == []


def test_task_table_set_get_pop():
    tt = TaskTable(4)
    tt.set("a", [3, 1], cached=4)
    assert tt.get("a") == [3, 1] and tt.get_cached("a") == 4
    assert tt.pop("a") == ([3, 1], 4) and tt.get("a") == []


def test_task_table_missing_task_is_empty():
    tt = TaskTable(4)
    assert tt.get("nope") == [] and tt.get_cached("nope") == 0


def test_task_table_tensor_pads_with_minus_one():
    tt = TaskTable(4)
    tt.set("a", [1], 0)
    tt.set("b", [2, 3, 4], 0)
    assert tt.table_tensor(["a", "b"], "cpu").tolist() == [[1, -1, -1], [2, 3, 4]]


def test_task_table_tensor_of_no_tasks():
    assert TaskTable(4).table_tensor([], "cpu").numel() == 0


# ---------------------------------------------------------------------------------------- tasks
class _Tok:
    stop_ids = [0]

    def encode(self, text):
        return [int(t) for t in text.split()] if text.strip() else []

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(i) for i in ids)


def test_new_task_is_pending():
    assert Task("t", [1, 2]).status is TaskStatus.PENDING


def test_task_next_pos_counts_prompt_and_outputs():
    t = Task("t", [5, 6, 7])
    t.output_ids = [9]
    assert t.next_pos == 3
    t.output_ids.append(4)
    assert t.next_pos == 4


def test_task_finishes_at_its_token_budget():
    t = Task("t", [1], max_tokens=2)
    t.output_tokens = 2
    assert t.is_finished([99])


def test_task_finishes_on_a_stop_id():
    t = Task("t", [1])
    t.output_ids = [3, 7]
    assert t.is_finished([7]) and not t.is_finished([3])


def test_task_history_window():
    t = Task("t", list(range(10)), rep_window=3)
    t.output_ids = [42]
    assert t.history() == [7, 8, 9, 42]


def test_manager_queues_and_counts_tasks():
    m = TaskManager(_Tok(), max_seq_len=64, max_prompt_len=16)
    tid = m.add_task("1 2 3")
    assert [t.task_id for t in m.get_waiting_tasks()] == [tid] and m.get_stats()["total_tasks"] == 1


def test_manager_answers_a_too_long_prompt_with_stop():
    got = []
    m = TaskManager(_Tok(), max_seq_len=4, max_prompt_len=0)
    m.add_task("1 2 3 4 5", stream_callback=got.append)
    assert got == [STOP] and not m.has_work()


def test_manager_keeps_the_prompt_tail():
    m = TaskManager(_Tok(), max_seq_len=64, max_prompt_len=2)
    m.add_task("1 2 3 4")
    assert m.get_waiting_tasks()[0].prompt_ids == [3, 4]


def test_manager_clamps_max_tokens_to_the_room_left():
    m = TaskManager(_Tok(), max_seq_len=10, max_prompt_len=8)
    m.add_task("1 2 3", max_tokens=100)
    assert m.get_waiting_tasks()[0].max_tokens == 7


def test_manager_pulls_in_fifo_order():
    m = TaskManager(_Tok())
    ids = [m.add_task(f"{i} 1") for i in range(4)]
    assert [t.task_id for t in m.pull_candidates(3)] == ids[:3]


def test_manager_return_to_waiting_restores_the_front():
    m = TaskManager(_Tok())
    ids = [m.add_task(f"{i} 1") for i in range(3)]
    got = m.pull_candidates(2)
    m.return_to_waiting(got)
    assert [t.task_id for t in m.get_waiting_tasks()] == ids


def test_manager_activate_and_remove_active():
    m = TaskManager(_Tok())
    tid = m.add_task("1 2")
    (t,) = m.pull_candidates(1)
    m.activate(t)
    assert t.status is TaskStatus.RUNNING and m.get_active_tasks() == [t]
    assert m.remove_task(tid) == [t] and not m.has_work()


def test_manager_remove_waiting_task():
    m = TaskManager(_Tok())
    tid = m.add_task("1 2")
    assert m.remove_task(tid) == [] and m.get_waiting_tasks() == []


def test_manager_retires_finished_and_aborted_tasks():
    m = TaskManager(_Tok())
    for s in ("1 2", "3 4", "5 6"):
        m.add_task(s, max_tokens=5)
    a, b, c = m.pull_candidates(3)
    for t in (a, b, c):
        m.activate(t)
    a.output_ids, a.output_tokens = [0], 1  # stop id
    b.status = TaskStatus.ABORTED
    done = m.remove_finished_tasks(_Tok.stop_ids)
    assert set(done) == {a, b} and a.status is TaskStatus.FINISHED and b.status is TaskStatus.ABORTED
    assert m.get_active_tasks() == [c] and m.get_stats()["total_tokens"] == 1


def test_manager_callbacks_reach_the_task():
    got = []
    m = TaskManager(_Tok())
    tid = m.add_task("1", stream_callback=got.append)
    m.invoke_callback(tid, "x")
    assert got == ["x"]


def test_manager_wait_returns_when_woken():
    m = TaskManager(_Tok())
    th = threading.Thread(target=lambda: m.wait_for_tasks(timeout=10.0))
    th.start()
    m.wake()
    th.join(timeout=5.0)
    assert not th.is_alive()


def test_manager_wait_returns_at_once_with_work():
    m = TaskManager(_Tok())
    m.add_task("1")
    m.wait_for_tasks(timeout=10.0)  # would block 10 s without work


# ---------------------------------------------------------------------------------------- engine results / requests
def test_result_collects_pieces_per_prompt():
    r = GenerateResult(2)
    for idx, piece in ((0, "a"), (1, "x"), (0, "b"), (0, STOP), (1, STOP)):
        r.append(piece, idx)
    assert list(r.events(timeout=1.0)) == [(0, "a"), (1, "x"), (0, "b")]
    assert r.get_results() == ["ab", "x"] and r.finished


def test_result_second_stop_of_a_prompt_is_harmless():
    r = GenerateResult(1)
    for piece in ("a", STOP, STOP):
        r.append(piece)
    assert list(r.events(timeout=1.0)) == [(0, "a")]


def test_result_times_out_when_nothing_arrives():
    r = GenerateResult(1)
    with pytest.raises(TimeoutError):
        list(r.events(timeout=0.2))


def test_result_events_from_another_thread():
    r = GenerateResult(1)

    def produce():
        for p in ("x", "y"):
            r.append(p)
        r.append(STOP)

    threading.Timer(0.1, produce).start()
    assert "".join(p for _, p in r.events(timeout=5.0)) == "xy"


@pytest.mark.parametrize("kw", [dict(top_p=1.5), dict(top_k=-1), dict(temperature=-0.1),
                                dict(frequency_penalty=3.0), dict(rep_window=0)])
def test_request_rejects_bad_sampling_parameters(kw):
    with pytest.raises(ValueError):
        GenerationRequest([{"role": "user", "content": "x"}], **kw)


def test_request_accepts_top_k_zero_and_greedy():
    r = GenerationRequest([{"role": "user", "content": "x"}], top_k=0, temperature=0.0)
    assert r.sampling()["top_k"] == 0 and r.sampling()["temperature"] == 0.0


# ---------------------------------------------------------------------------------------- detokeniser
class _Bytes:
    def decode(self, ids, skip_special_tokens=True):
        return bytes(ids).decode("utf-8", errors="replace")


def test_stream_decoder_emits_ascii_at_once():
    d = StreamDecoder(_Bytes())
    assert "".join(d.push(b) for b in b"hello") == "hello"


def test_stream_decoder_holds_split_multibyte_characters():
    d = StreamDecoder(_Bytes())
    out = [d.push(b) for b in "é✓".encode()]
    assert "".join(out) == "é✓" and out[0] == "" and out[2] == ""


def test_stream_decoder_flush_releases_a_dangling_byte():
    d = StreamDecoder(_Bytes())
    d.push(ord("a"))
    d.push(0xE2)
    assert d.flush().startswith("�") or d.flush() == ""


def test_stream_decoder_keeps_spaces_between_words():
    class Words:
        vocab = {1: "the", 2: "quick", 3: "fox"}

        def decode(self, ids, skip_special_tokens=True):
            return " ".join(self.vocab[i] for i in ids)

    d = StreamDecoder(Words())
    assert "".join(d.push(i) for i in (1, 2, 3)) == "the quick fox"


# ---------------------------------------------------------------------------------------- sampling strategies
def test_temperature_divides_logits():
    x = torch.tensor([[1.0, 2.0]])
    assert torch.allclose(TemperatureStrategy(0.5).apply(x), x * 2)


def test_temperature_one_is_a_no_op():
    x = torch.randn(2, 5)
    assert TemperatureStrategy(1.0).apply(x) is x


def test_temperature_per_row():
    x = torch.ones(2, 3)
    out = TemperatureStrategy(torch.tensor([1.0, 0.5])).apply(x)
    assert torch.allclose(out[1], torch.full((3,), 2.0))


def test_top_k_keeps_the_k_largest():
    x = torch.tensor([[1.0, 5.0, 3.0, 4.0]])
    out = TopKStrategy(2).apply(x)
    assert torch.isinf(out[0, [0, 2]]).all() and torch.equal(out[0, [1, 3]], x[0, [1, 3]])


def test_top_k_zero_keeps_everything():
    x = torch.randn(3, 6)
    assert torch.equal(TopKStrategy(0).apply(x), x)


def test_top_k_per_row():
    x = torch.arange(8.0).repeat(2, 1)
    out = TopKStrategy(torch.tensor([1, 3])).apply(x)
    assert torch.isfinite(out[0]).sum() == 1 and torch.isfinite(out[1]).sum() == 3


def test_top_p_keeps_the_nucleus():
    x = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]]))
    out = TopPStrategy(0.7).apply(x)
    assert torch.isfinite(out[0, :2]).all() and torch.isinf(out[0, 2:]).all()


def test_top_p_one_is_a_no_op():
    x = torch.randn(2, 4)
    assert torch.equal(TopPStrategy(1.0).apply(x), x)


def test_top_p_zero_keeps_only_the_best():
    x = torch.tensor([[0.1, 2.0, 0.3]])
    assert torch.isfinite(TopPStrategy(0.0).apply(x)).sum() == 1


def test_frequency_penalty_counts_occurrences():
    x = torch.zeros(1, 5)
    out = FrequencyPenaltyStrategy(0.5).apply(x, input_ids=torch.tensor([[1, 1, 3]]))
    assert out[0].tolist() == [0.0, -1.0, 0.0, -0.5, 0.0]


def test_frequency_penalty_respects_the_mask():
    x = torch.zeros(1, 4)
    out = FrequencyPenaltyStrategy(1.0).apply(x, input_ids=torch.tensor([[2, 2]]),
                                              input_mask=torch.tensor([[True, False]]))
    assert out[0, 2].item() == -1.0


def test_negative_frequency_penalty_boosts_repeats():
    out = FrequencyPenaltyStrategy(-1.0).apply(torch.zeros(1, 3), input_ids=torch.tensor([[0]]))
    assert out[0, 0].item() == 1.0


def test_frequency_penalty_without_history_is_a_no_op():
    x = torch.randn(1, 3)
    assert FrequencyPenaltyStrategy(1.0).apply(x) is x


def test_pipeline_applies_strategies_in_order():
    x = torch.tensor([[1.0, 2.0, 3.0, 4.0]])
    out = SamplingPipeline([TemperatureStrategy(2.0), TopKStrategy(1)]).apply(x)
    assert torch.isfinite(out).sum() == 1 and out[0, 3].item() == 2.0


def test_sample_returns_a_token_per_row():
    tok = sample(torch.randn(5, 11), temperature=0.8, top_k=4)
    assert tok.shape == (5,) and (tok >= 0).all() and (tok < 11).all()


def test_greedy_sample_is_argmax():
    x = torch.randn(4, 9)
    assert torch.equal(sample(x, temperature=0.0), x.argmax(-1))


def test_sample_logprobs_are_log_probabilities():
    x = torch.randn(3, 7)
    tok, lp = sample(x, temperature=1.0, return_logprobs=True)
    ref = torch.log_softmax(x, -1).gather(-1, tok[:, None]).squeeze(-1)
    assert torch.allclose(lp, ref, atol=1e-5) and (lp <= 0).all()


def test_sample_respects_top_k_one():
    x = torch.randn(6, 20)
    assert torch.equal(sample(x, temperature=1.0, top_k=1), x.argmax(-1))


# ---------------------------------------------------------------------------------------- stop sequences / builders
def test_stop_checker_finds_the_earliest_sequence():
    assert StopChecker(["END", "x"]).check("abxEND") == "x"


def test_stop_checker_without_match():
    assert StopChecker(["END"]).check("hello") is None


def test_stop_checker_without_sequences_emits_everything():
    assert StopChecker([]).cut("abc</") == (None, "abc</")


def test_stop_checker_holds_back_a_possible_prefix():
    assert StopChecker(["</s>"]).cut("hi </") == (None, "hi ")


class _Msg:
    def __init__(self, role, content):
        self.role, self.content = role, content
        self.tool_calls = self.tool_call_id = None


class _OpenAIReq:
    def __init__(self, **kw):
        self.messages = kw.get("messages", [_Msg("user", "hi")])
        self.model = "m"
        self.max_tokens = kw.get("max_tokens")
        self.stop = kw.get("stop")
        self.tools = kw.get("tools")
        self.tool_choice = "auto"
        self.stream = False


class _TmplTok:
    def apply_chat_template(self, messages, tokenize=False, **kw):
        return "".join(f"<{m['role']}>{m['content']}" for m in messages)

    def encode(self, text):
        return list(text.encode())


class _StubEngine:
    tokenizer = _TmplTok()


def parse_sse(events):
    return [json.loads(e.split("data: ", 1)[1]) for e in events if "data: {" in e]


def test_openai_prepare_renders_the_template_and_stops():
    from astrai_b200.inference.api.openai import OpenAIResponseBuilder

    prompt, ctx, stops = OpenAIResponseBuilder().prepare(_OpenAIReq(stop="END"), _StubEngine())
    assert prompt == "<user>hi" and stops == ["END"] and ctx.resp_id.startswith("chatcmpl-")


def test_openai_stream_events():
    from astrai_b200.inference.api.openai import OpenAIResponseBuilder

    b = OpenAIResponseBuilder()
    _, ctx, _ = b.prepare(_OpenAIReq(), _StubEngine())
    ev = b.format_stream_start(ctx) + b.format_chunk("Hel") + b.format_chunk("lo")
    ctx.completion_tokens = 2
    ev += b.format_stream_end(ctx, StopInfo(None, "Hello", "Hello"))
    data = parse_sse(ev)
    assert data[0]["choices"][0]["delta"] == {"role": "assistant"}
    assert "".join(d["choices"][0]["delta"].get("content", "") for d in data) == "Hello"
    assert data[-1]["choices"][0]["finish_reason"] == "stop" and data[-1]["usage"]["completion_tokens"] == 2


def test_openai_finish_reason_length():
    from astrai_b200.inference.api.openai import OpenAIResponseBuilder

    b = OpenAIResponseBuilder()
    _, ctx, _ = b.prepare(_OpenAIReq(max_tokens=3), _StubEngine())
    ctx.completion_tokens = 3
    assert b.format_response(ctx, "abc", StopInfo())["choices"][0]["finish_reason"] == "length"


def test_openai_response_with_tool_call():
    from astrai_b200.inference.api.openai import OpenAIResponseBuilder

    tools = [{"type": "function", "function": {"name": "f", "parameters": {}}}]
    b = OpenAIResponseBuilder()
    _, ctx, _ = b.prepare(_OpenAIReq(tools=tools), _StubEngine())
    r = b.format_response(ctx, '{"name": "f", "arguments": {"a": 1}}', StopInfo())
    msg = r["choices"][0]["message"]
    assert r["choices"][0]["finish_reason"] == "tool_calls" and msg["tool_calls"][0]["function"]["name"] == "f"


class _AnthReq:
    def __init__(self, system=None, stop_sequences=None, max_tokens=16):
        self.messages = [_Msg("user", [{"type": "text", "text": "hey"}])]
        self.system, self.stop_sequences, self.max_tokens, self.model = system, stop_sequences, max_tokens, "m"


def test_anthropic_prepare_puts_the_system_prompt_first():
    from astrai_b200.inference.api.anthropic import AnthropicResponseBuilder

    prompt, ctx, stops = AnthropicResponseBuilder().prepare(_AnthReq(system="be brief", stop_sequences=["\n\n"]),
                                                            _StubEngine())
    assert prompt == "<system>be brief<user>hey" and stops == ["\n\n"] and ctx.resp_id.startswith("msg_")


def test_anthropic_stream_event_sequence():
    from astrai_b200.inference.api.anthropic import AnthropicResponseBuilder

    b = AnthropicResponseBuilder()
    _, ctx, _ = b.prepare(_AnthReq(), _StubEngine())
    ev = b.format_stream_start(ctx) + b.format_chunk("yo") + b.format_stream_end(ctx, StopInfo("STOP", "yo", "yo"))
    types = [d["type"] for d in parse_sse(ev)]
    assert types == ["message_start", "content_block_start", "content_block_delta", "content_block_stop",
                     "message_delta", "message_stop"]
    assert parse_sse(ev)[4]["delta"]["stop_reason"] == "stop_sequence"


def test_anthropic_response_end_turn():
    from astrai_b200.inference.api.anthropic import AnthropicResponseBuilder

    b = AnthropicResponseBuilder()
    _, ctx, _ = b.prepare(_AnthReq(max_tokens=100), _StubEngine())
    r = b.format_response(ctx, "done", StopInfo())
    assert r["stop_reason"] == "end_turn" and r["content"] == [{"type": "text", "text": "done"}]


# ---------------------------------------------------------------------------------------- HTTP server (stub engine)
class _ServerEngine:
    tokenizer = _TmplTok()

    def __init__(self, pieces):
        self.pieces = pieces

    def generate_async(self, prompt, **kw):
        pieces = self.pieces

        async def agen():
            for p in pieces:
                await asyncio.sleep(0)
                yield p

        return agen()

    def get_stats(self):
        return {"total_tasks": 0}


@pytest.fixture
def client():
    from starlette.testclient import TestClient

    from astrai_b200.inference.api.server import get_app

    app = get_app()
    app.state.engine = None
    app.state.server_config = {}
    with TestClient(app) as c:
        yield app, c
    app.state.engine = None


def test_health_without_a_model(client):
    _, c = client
    assert c.get("/health").json() == {"status": "ok", "model_loaded": False}


def test_endpoints_need_an_engine(client):
    _, c = client
    assert c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}]}).status_code == 503


def test_chat_completion_non_streaming(client):
    app, c = client
    app.state.engine = _ServerEngine(["Hel", "lo"])
    r = c.post("/v1/chat/completions", json={"model": "m", "messages": [{"role": "user", "content": "x"}]}).json()
    assert r["choices"][0]["message"]["content"] == "Hello" and r["object"] == "chat.completion"


def test_chat_completion_streaming(client):
    app, c = client
    app.state.engine = _ServerEngine(["a", "b", "c"])
    body = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                "stream": True}).text
    chunks = [json.loads(line[6:]) for line in body.splitlines() if line.startswith("data: {")]
    assert "".join(ch["choices"][0]["delta"].get("content", "") for ch in chunks) == "abc"
    assert body.rstrip().endswith("data: [DONE]")


def test_chat_completion_stop_sequence(client):
    app, c = client
    app.state.engine = _ServerEngine(["one ", "two", " STOP three"])
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "stop": ["STOP"]}).json()
    assert r["choices"][0]["message"]["content"] == "one two " and r["choices"][0]["finish_reason"] == "stop"


def test_chat_completion_stop_sequence_streaming(client):
    app, c = client
    app.state.engine = _ServerEngine(["one ", "tw", "o ST", "OP more"])
    body = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "stop": "STOP",
                                                "stream": True}).text
    chunks = [json.loads(line[6:]) for line in body.splitlines() if line.startswith("data: {")]
    assert "".join(ch["choices"][0]["delta"].get("content", "") for ch in chunks) == "one two "


def test_messages_non_streaming_with_system(client):
    app, c = client
    app.state.engine = _ServerEngine(["fine"])
    r = c.post("/v1/messages", json={"model": "m", "max_tokens": 8, "system": "s",
                                     "messages": [{"role": "user", "content": "hi"}]}).json()
    assert r["content"][0]["text"] == "fine" and r["type"] == "message"


def test_messages_streaming(client):
    app, c = client
    app.state.engine = _ServerEngine(["x", "y"])
    body = c.post("/v1/messages", json={"model": "m", "max_tokens": 8, "stream": True,
                                        "messages": [{"role": "user", "content": "hi"}]}).text
    events = [line[7:] for line in body.splitlines() if line.startswith("event: ")]
    assert events[0] == "message_start" and events[-1] == "message_stop"


# ---------------------------------------------------------------------------------------- scheduler threads
def _tiny_scheduler():
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.inference.core.scheduler import InferenceScheduler
    from astrai_b200.models import AutoRegressiveLM

    torch.manual_seed(0)
    m = AutoRegressiveLM(AutoRegressiveLMConfig(vocab_size=64, hidden_size=32, num_hidden_layers=1, rms_norm_eps=1e-5,
                                                intermediate_size=64, max_position_embeddings=64, rope_theta=1e4,
                                                num_attention_heads=2, num_key_value_heads=1)).eval()

    class Tok(_Tok):
        stop_ids = []

    return InferenceScheduler(m, Tok(), max_batch_size=4, max_seq_len=48, max_prompt_len=16)


def test_scheduler_concurrent_add_and_remove():
    sch = _tiny_scheduler()
    ids, lock = [], threading.Lock()

    def worker(k):
        for i in range(20):
            tid = sch.add_task(f"{k} {i} 1", max_tokens=2)
            with lock:
                ids.append(tid)
            if i % 2:
                sch.remove_task(tid)

    threads = [threading.Thread(target=worker, args=(k,)) for k in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert len(set(ids)) == 80 and sch.get_stats()["total_tasks"] == 80


def test_scheduler_stats_are_readable_while_adding():
    sch = _tiny_scheduler()
    stop = threading.Event()
    seen = []

    def reader():
        while not stop.is_set():
            seen.append(sch.get_stats()["total_tasks"])

    th = threading.Thread(target=reader)
    th.start()
    for i in range(50):
        sch.add_task(f"{i} 2")
    stop.set()
    th.join()
    assert seen == sorted(seen) and sch.get_stats()["total_tasks"] == 50


def test_run_batch_respects_max_tokens_and_empty_prompts():
    sch = _tiny_scheduler()
    out = sch.run_batch([[1, 2, 3], [], [4, 5]], max_tokens=3, temperature=0.0)
    assert [len(o) for o in out] == [3, 0, 3]


def test_run_batch_skips_prompts_longer_than_the_context():
    sch = _tiny_scheduler()
    assert sch.run_batch([list(range(1, 60))], max_tokens=2) == [[]]


def test_run_batch_logprobs_align_with_tokens():
    sch = _tiny_scheduler()
    (toks, lps), = sch.run_batch([[3, 4, 5]], max_tokens=4, temperature=1.0, return_logprobs=True)
    assert len(toks) == len(lps) == 4 and all(lp <= 0 for lp in lps)
