"""Evaluation suite on CPU: the packed scorer against one plain forward per document, and the
text-only metrics (ROUGE, pass@k, IFEval verifiers, SVD ranks) against hand-computed values."""

import json
import math
import os

import pytest
import torch

from tests.conftest import TINY_CFG, make_tokenizer_files


@pytest.fixture(scope="module")
def model():
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM

    torch.manual_seed(0)
    return AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG)).float().eval()


def _plain_logprobs(model, ids, n_ctx):
    x = torch.tensor([ids])
    lp = torch.log_softmax(model(x)["logits"][0].float(), -1)
    return torch.stack([lp[p - 1, ids[p]] for p in range(n_ctx, len(ids))])


def test_packed_scorer_matches_one_forward_per_document(model):
    from astrai_b200.eval.loglik import Doc, score_docs

    g = torch.Generator().manual_seed(1)
    docs = [Doc(torch.randint(0, 512, (n,), generator=g).tolist(), c) for n, c in
            [(17, 5), (40, 1), (9, 8), (64, 30), (23, 2), (5, 1)]]
    got = score_docs(model, docs, max_len=64, max_tokens=128)
    for d, lp in zip(docs, got):
        ref = _plain_logprobs(model, d.ids, d.n_ctx)
        assert lp.shape == ref.shape
        torch.testing.assert_close(lp, ref, atol=2e-4, rtol=1e-4)


def test_next_token_logprobs_and_fit(model):
    from astrai_b200.eval.loglik import fit, next_token_logprobs

    ctxs = [[1, 2, 3, 4], [7, 8], list(range(10, 40))]
    lsm = next_token_logprobs(model, ctxs, max_len=32)
    for c, row in zip(ctxs, lsm):
        ref = torch.log_softmax(model(torch.tensor([c]))["logits"][0, -1].float(), -1)
        torch.testing.assert_close(row, ref, atol=2e-4, rtol=1e-4)
    d = fit(list(range(100)), [1, 2, 3], 10)
    assert d.ids == list(range(93, 100)) + [1, 2, 3] and d.n_ctx == 7


def test_ppl_ifd_mmlu_end_to_end(tmp_path, model):
    from astrai_b200.eval import ifd, mmlu, ppl
    from astrai_b200.tokenize import AutoTokenizer

    make_tokenizer_files(str(tmp_path / "tok"))
    tok = AutoTokenizer.from_pretrained(str(tmp_path / "tok"))
    texts = ["hello world, this is a tiny corpus", "the quick brown fox jumps over the lazy dog"]
    st = ppl.evaluate_texts(model, tok, texts, max_length=64, token_level=True)
    n = sum(len(tok.encode(t)) - 1 for t in texts)
    assert st["overall"]["num_tokens"] == n and math.isclose(st["overall"]["ppl"],
                                                             math.exp(st["overall"]["mean_loss"]))
    assert sum(v["num_tokens"] for v in st["by_token_type"].values()) == n
    rows = ifd.score_items(model, tok, [{"instruction": "say hello", "response": "hello world"},
                                        {"instruction": "", "response": "x"}], max_len=64)
    assert rows[0]["ifd"] == pytest.approx(rows[0]["ifd_detail"]["L_cond"] / rows[0]["ifd_detail"]["L_uncond"],
                                           rel=1e-4)
    assert rows[1]["ifd"] is None
    d = tmp_path / "mmlu" / "test"
    d.mkdir(parents=True)
    with open(d / "toy_test.csv", "w") as fh:
        fh.write('q1,A)one,B)two,C)three,D)four,B\nq2,a,b,c,d,D\n')
    res = mmlu.run(model, tok, str(tmp_path / "mmlu"), "test", n_shot=0)
    assert res["_overall"]["total"] == 2 and "toy" in res


def test_rouge_values():
    from astrai_b200.eval.rouge import compute_rouge, lcs_len

    s = compute_rouge("the cat sat on the mat", "the cat on the mat")
    assert s["rouge-1"]["precision"] == 1.0 and s["rouge-1"]["recall"] == pytest.approx(5 / 6)
    assert s["rouge-2"]["precision"] == pytest.approx(3 / 4)
    assert lcs_len("a b c d".split(), "a c d".split()) == 3


def test_pass_at_k_and_extraction():
    from astrai_b200.eval.humaneval import extract_body, pass_at_k, program, trim_stop

    assert pass_at_k(10, 0, 1) == 0.0 and pass_at_k(10, 10, 5) == 1.0
    assert pass_at_k(5, 2, 1) == pytest.approx(0.4)
    assert pass_at_k(5, 2, 2) == pytest.approx(1 - math.comb(3, 2) / math.comb(5, 2))
    assert trim_stop("    return 1\ndef other():\n") == "    return 1"
    assert extract_body("def f(x):\n    return x\nprint(1)", "f") == "    return x"
    code = program({"prompt": "def f(x):\n", "test": "def check(c):\n    assert c(2) == 2\n", "entry_point": "f"},
                   "    return x")
    assert code.rstrip().endswith("check(f)")


def test_ifeval_verifiers():
    from astrai_b200.eval.ifeval import score, verify

    assert verify("I LOVE IT", "change_case:english_capital", {})
    assert verify("no commas here", "punctuation:no_comma", {})
    assert not verify("a, b", "punctuation:no_comma", {})
    assert verify("* a\n* b\n- c", "detectable_format:number_bullet_lists", {"num_bullets": 3})
    assert verify('{"a": 1}', "detectable_format:json_format", {})
    assert verify("```json\n{\"a\": 1}\n```", "detectable_format:json_format", {})
    assert verify("one two three", "length_constraints:number_words", {"num_words": 4, "relation": "less than"})
    assert verify("<<Title>> body", "detectable_format:title", {})
    assert verify("p1\n\np2", "length_constraints:number_paragraphs", {"num_paragraphs": 2})
    assert verify("x ****** y", "combination:two_responses", {})
    assert verify("anything", "language:response_language", {"language": "en"}) is None
    res = score([{"key": 1, "prompt": "p", "instruction_id_list": ["punctuation:no_comma", "language:response_language"],
                  "kwargs": [{}, {"language": "en"}]}], [["a, b", "ab"]])
    assert res["1"]["num_passed"] == 1 and res["_summary"]["unsupported_constraints"] == 1


def test_weight_analysis_ranks():
    from astrai_b200.eval.weights import analyze

    torch.manual_seed(0)
    u = torch.linalg.qr(torch.randn(32, 32))[0]
    low = (u[:, :4] * torch.tensor([8.0, 4.0, 2.0, 1.0])) @ torch.linalg.qr(torch.randn(16, 4))[0].T  # rank 4
    res = analyze({"layers.0.attention.q_proj.weight": low, "layers.1.attention.q_proj.weight": torch.eye(32)[:, :16],
                   "norm.weight": torch.ones(16)}, device="cpu")
    assert res["layers.0.attention.q_proj.weight"]["er_99"] == 4
    assert res["layers.1.attention.q_proj.weight"]["entropic_rank"] == pytest.approx(16, rel=1e-6)
    assert res["norm.weight"]["is_1d"]


def test_demos_and_generation_evals_on_cpu_engine(tmp_path, model):
    from astrai_b200.demo.batch import batch_generate
    from astrai_b200.demo.chat import chat
    from astrai_b200.demo.generate import generate_text
    from astrai_b200.eval.ifeval import evaluate
    from astrai_b200.inference import InferenceEngine
    from astrai_b200.tokenize import AutoTokenizer

    make_tokenizer_files(str(tmp_path / "tok"))
    tok = AutoTokenizer.from_pretrained(str(tmp_path / "tok"))
    with InferenceEngine(model, tok, max_batch_size=2, max_seq_len=96) as eng:
        assert len(chat(["--max_tokens", "4"], queries=["hello", "!exit"], engine=eng, tokenizer=tok)) == 1
        assert len(batch_generate(["--max_tokens", "4", "--queries", "a", "b", "c"], engine=eng, tokenizer=tok)) == 3
        assert isinstance(generate_text(["--max_tokens", "4"], prompt="hello", engine=eng), str)
        res = evaluate(eng, tok, [{"key": 7, "prompt": "hi", "instruction_id_list": ["punctuation:no_comma"],
                                   "kwargs": [{}]}], max_tokens=4, num_samples=2)
        assert res["7"]["num_samples"] == 2 and res["_summary"]["total_constraints"] == 1
