"""Inference kernels and the generation path on the GPU.

Paged KV write / gather and the split-KV decode kernel against plain fp32
PyTorch over the same pages; the fused sampler against the strategy
pipeline (exact for greedy / top-k=1, support and log-probabilities for the
filtered cases, frequencies for the draw); decode-step consistency of the
engine (eager and CUDA graph) with a full forward pass.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_error_word():
    from astrai_b200.ops._ext import native

    native().read_error()
    yield
    torch.cuda.synchronize()
    assert native().read_error() == 0


def _rand_cache(n_pages, Hkv, page, seed=0, D=128):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(n_pages, Hkv, page, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(n_pages, Hkv, page, D, device="cuda", generator=g).to(torch.bfloat16)
    return kc, vc


def _gather_ref(kc, vc, table, lens, total):
    B = table.shape[0]
    page = kc.shape[2]
    k = torch.zeros(B, total, kc.shape[1], kc.shape[3], device="cuda", dtype=torch.float32)
    v = torch.zeros_like(k)
    for b in range(B):
        for p in range(int(lens[b])):
            pg = int(table[b, p // page])
            if pg >= 0:
                k[b, p] = kc[pg, :, p % page].float()
                v[b, p] = vc[pg, :, p % page].float()
    return k, v


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("page", [16, 128])
def test_paged_write_and_gather(page, D):
    from astrai_b200.ops._ext import native

    C = native()
    Hkv, n_pages = 2, 12
    kc, vc = _rand_cache(n_pages, Hkv, page, D=D)
    T = 3 * page // 2
    qkv = torch.randn(T, (4 + 2 * Hkv) * D, device="cuda").to(torch.bfloat16)
    k = qkv[:, 4 * D:(4 + Hkv) * D]
    v = qkv[:, (4 + Hkv) * D:]
    pages = torch.tensor([7, 3], device="cuda")
    pos = torch.arange(T, device="cuda")
    slots = (pages[pos // page] * page + pos % page).to(torch.int32)
    slots[5] = -1  # skipped row
    kc0 = kc.clone()
    C.paged_kv_write(k, v, slots, kc, vc)
    torch.cuda.synchronize()
    for t in (0, 5, T - 1):
        pg, off = int(pages[t // page]), t % page
        want_k = kc0[pg, :, off] if t == 5 else k[t].view(Hkv, D)
        assert torch.equal(kc[pg, :, off], want_k)
        if t != 5:
            assert torch.equal(vc[pg, :, off], v[t].view(Hkv, D))
    table = torch.tensor([[7, 3, -1], [3, -1, -1]], device="cuda", dtype=torch.int32)
    lens = torch.tensor([T, page // 2], device="cuda", dtype=torch.int32)
    ko, vo = C.paged_kv_gather(kc, vc, table, lens, 2 * page)
    kr, vr = _gather_ref(kc, vc, table, lens, 2 * page)
    assert torch.equal(ko.float(), kr) and torch.equal(vo.float(), vr)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("G", [1, 2, 3, 4, 6, 8, 12, 16])
@pytest.mark.parametrize("page,lens", [(16, [1, 17, 300, 64]), (64, [65, 700, 3, 128]),
                                       (128, [513, 128, 5, 1000]), (256, [257, 1, 900, 256])])
@pytest.mark.parametrize("splits", [1, 7])
def test_paged_decode_matches_reference(G, page, lens, splits, D):
    from astrai_b200.ops._ext import native

    C = native()
    torch.manual_seed(G)
    Hkv, B = 2, len(lens)
    Hq = G * Hkv
    max_pages = max(-(-L // page) for L in lens)
    n_pages = B * max_pages + 3
    kc, vc = _rand_cache(n_pages, Hkv, page, seed=G, D=D)
    perm = torch.randperm(n_pages)[: B * max_pages].view(B, max_pages)
    table = perm.to(torch.int32).cuda()
    for b, L in enumerate(lens):
        table[b, -(-L // page):] = -1
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq * D, device="cuda").to(torch.bfloat16)
    out = torch.empty(B, Hq * D, device="cuda", dtype=torch.bfloat16)
    ws = torch.empty(B * Hq * splits * (D + 2), device="cuda", dtype=torch.float32)
    scale = 1 / math.sqrt(D)
    C.paged_decode(q, kc, vc, table, ln, out, Hq, scale, splits, ws)
    kr, vr = _gather_ref(kc, vc, table, ln, max(lens))
    for b, L in enumerate(lens):
        qb = q[b].view(Hq, D).float()
        kb = kr[b, :L].repeat_interleave(G, dim=1)  # [L, Hq, D]
        vb = vr[b, :L].repeat_interleave(G, dim=1)
        s = torch.einsum("hd,lhd->hl", qb, kb) * scale
        o = torch.einsum("hl,lhd->hd", torch.softmax(s, -1), vb)
        torch.testing.assert_close(out[b].view(Hq, D).float(), o, atol=2e-2, rtol=2e-2)


def _logits(rows, V, seed=0, spread=3.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(rows, V, device="cuda", generator=g) * spread)


@pytest.mark.parametrize("V", [512, 16384, 32000, 151936])
def test_sample_greedy_and_topk1(V):
    from astrai_b200.inference.sample import sample

    x = _logits(8, V, seed=V)
    tok, lp = sample(x, temperature=0.0, return_logprobs=True)
    assert torch.equal(tok, x.argmax(-1))
    torch.testing.assert_close(lp, torch.log_softmax(x, -1).gather(1, tok[:, None]).squeeze(1), atol=1e-4, rtol=1e-4)
    xb = x.to(torch.bfloat16)
    tok2 = sample(xb, temperature=0.7, top_k=1)  # ties at the maximum all survive top-k (as in the reference)
    assert torch.equal(xb.gather(1, tok2[:, None]).squeeze(1), xb.max(-1).values)


@pytest.mark.parametrize("V", [1000, 32000])
def test_sample_topk_topp_support_and_logprob(V):
    from astrai_b200.inference.sample import (SamplingPipeline, TemperatureStrategy, TopKStrategy, TopPStrategy,
                                              sample)

    rows = 64
    x = _logits(rows, V, seed=1)
    temp = torch.full((rows,), 0.8, device="cuda")
    topk = torch.randint(1, 60, (rows,), device="cuda")
    topp = torch.rand(rows, device="cuda") * 0.9 + 0.05
    tok, lp = sample(x, temperature=temp, top_k=topk, top_p=topp, return_logprobs=True)
    ref = SamplingPipeline([TemperatureStrategy(temp), TopKStrategy(topk), TopPStrategy(topp)]).apply(x.clone())
    ref_lp = torch.log_softmax(ref, -1)
    chosen = ref_lp.gather(1, tok[:, None]).squeeze(1)
    assert torch.isfinite(chosen).all(), "sampled a token outside the filtered support"
    torch.testing.assert_close(lp, chosen, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("V", [1000, 32000])
def test_sample_topp_only_support_and_logprob(V):
    """Top-p over the whole vocabulary (no top-k): the mass histogram and the exact in-bin cut."""
    from astrai_b200.inference.sample import SamplingPipeline, TemperatureStrategy, TopPStrategy, sample

    rows = 64
    x = _logits(rows, V, seed=4)
    temp = torch.full((rows,), 0.9, device="cuda")
    topp = torch.rand(rows, device="cuda") * 0.9 + 0.05
    tok, lp = sample(x, temperature=temp, top_k=0, top_p=topp, return_logprobs=True)
    ref = SamplingPipeline([TemperatureStrategy(temp), TopPStrategy(topp)]).apply(x.clone())
    chosen = torch.log_softmax(ref, -1).gather(1, tok[:, None]).squeeze(1)
    assert torch.isfinite(chosen).all(), "sampled a token outside the nucleus"
    torch.testing.assert_close(lp, chosen, atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("V", [4096, 32000])
def test_sample_massive_ties_keep_every_tied_token(V):
    """Every logit equal: one histogram bin holds the whole row, so the thresholds come from the
    in-bin bisection; ties at the threshold are all kept, so every token stays possible."""
    from astrai_b200.inference.sample import sample

    rows = 256
    x = torch.zeros(rows, V, device="cuda")
    for kw in (dict(top_k=50), dict(top_p=0.5), dict(top_k=50, top_p=0.5)):
        tok, lp = sample(x, temperature=1.0, return_logprobs=True, **kw)
        assert ((tok >= 0) & (tok < V)).all()
        torch.testing.assert_close(lp, torch.full_like(lp, -math.log(V)), atol=1e-3, rtol=1e-3)
        assert tok.unique().numel() > rows // 2  # spread over the tied tokens, not stuck on a few


def test_sample_frequency_penalty_logprob():
    from astrai_b200.inference.sample import FrequencyPenaltyStrategy, sample

    rows, V = 16, 4096
    x = _logits(rows, V, seed=2, spread=1.0)
    hist = torch.randint(0, 50, (rows, 40), device="cuda")
    mask = torch.rand(rows, 40, device="cuda") > 0.2
    pen = torch.full((rows,), 1.5, device="cuda")
    tok, lp = sample(x, temperature=1.0, top_k=0, frequency_penalty=pen, input_ids=hist, input_mask=mask,
                     return_logprobs=True)
    ref = FrequencyPenaltyStrategy(pen).apply(x.clone(), input_ids=hist, input_mask=mask)
    torch.testing.assert_close(lp, torch.log_softmax(ref, -1).gather(1, tok[:, None]).squeeze(1), atol=2e-3,
                               rtol=2e-3)


def test_sample_distribution_matches_softmax():
    from astrai_b200.inference.sample import sample

    V, rows = 6, 1 << 16
    base = torch.tensor([2.0, 1.0, 0.5, 0.0, -1.0, 0.3], device="cuda")
    x = base.expand(rows, V).contiguous()
    counts = torch.zeros(V, device="cuda")
    for _ in range(4):
        counts += torch.bincount(sample(x, temperature=1.0, top_k=0), minlength=V).float()
    freq = counts / counts.sum()
    assert (freq - torch.softmax(base, 0)).abs().max() < 5e-3
    k3 = torch.bincount(sample(x, temperature=1.0, top_k=3), minlength=V).float()
    assert k3[3:].sum() == 0  # top-3 = tokens 0, 1, 2
    p3 = torch.softmax(base[:3], 0)
    torch.testing.assert_close(k3[:3] / rows, p3, atol=1e-2, rtol=0)


def _gpu_model(seed=0, layers=2, vocab=2048, heads=2, kv=1, head_dim=128):
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM

    torch.manual_seed(seed)
    cfg = AutoRegressiveLMConfig(vocab_size=vocab, hidden_size=head_dim * heads, num_attention_heads=heads,
                                 num_key_value_heads=kv, intermediate_size=384, num_hidden_layers=layers,
                                 max_position_embeddings=512, rms_norm_eps=1e-5, rope_theta=10000.0)
    m = AutoRegressiveLM(cfg).cuda().to(torch.bfloat16).eval()
    with torch.no_grad():
        m.lm_head.weight.mul_(30.0)  # spread the logits so greedy choices are stable in bf16
    return m


class _Tok:
    stop_ids = [1]

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(i) for i in ids)

    def encode(self, s):
        return [int(x) for x in s.split()]


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("paged", [False, True])
def test_generation_matches_full_forward(graph, paged, head_dim):
    """Prefill (flash forward), decode (paged split-KV kernel) and the sampler against a full forward pass;
    head_dim 64 is the reference's benchmark model's head size (d 1536 over 24 heads)."""
    from astrai_b200.inference.core import InferenceScheduler, PageCache

    m = _gpu_model(heads=4, kv=2, head_dim=head_dim)
    cache = PageCache(2, 64, 16, 2, head_dim, "cuda", torch.bfloat16) if paged else None
    sch = InferenceScheduler(m, _Tok(), max_batch_size=4, max_seq_len=256, cache=cache, use_cuda_graph=graph)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(2, 2048, (n,), generator=g).tolist() for n in (5, 37, 16, 100)]
    out = sch.run_batch(prompts, max_tokens=12, temperature=0.0, return_logprobs=True)
    with torch.no_grad():
        for p, (toks, lps) in zip(prompts, out):
            assert 1 <= len(toks) <= 12
            seq = torch.tensor([p + toks], device="cuda")
            ref = torch.log_softmax(m(seq)["logits"][0].float(), -1)[len(p) - 1:len(p) - 1 + len(toks)]
            ref_tok = ref.gather(1, torch.tensor(toks, device="cuda")[:, None]).squeeze(1)
            # each generated token is (within bf16 noise) the argmax of the full forward pass: logits of
            # magnitude 16 - 40 are spaced 0.125 - 0.25 apart in bf16, so near-ties may flip by one step
            assert (ref.max(-1).values - ref_tok).max() <= 0.26
            # logits are O(30) here: bf16 rounding alone moves a log-probability by ~0.1
            torch.testing.assert_close(torch.tensor(lps, device="cuda"), ref_tok, atol=0.25, rtol=0.05)
    if paged:  # a second run over the same prompts reuses full prompt pages
        out2 = sch.run_batch(prompts, max_tokens=12, temperature=0.0)
        assert [len(o) for o in out2] == [len(o[0]) for o in out]


def test_engine_stream_and_batch():
    from astrai_b200.inference.engine import InferenceEngine

    m = _gpu_model()
    with InferenceEngine(m, _Tok(), max_batch_size=3, max_seq_len=128) as eng:
        pieces = list(eng.generate("5 6 7 8", stream=True, max_tokens=5, temperature=0.0))
        assert len(pieces) >= 1
        full = eng.generate(["5 6 7 8", "9 10"], max_tokens=5, temperature=0.0)
        assert full[0] == "".join(pieces)
        assert eng.get_stats()["total_tasks"] == 3


def test_extension_native_paths_match_reference():
    from astrai_b200.extension import attn_decode, attn_paged_decode, attn_prefill, reference_attention

    torch.manual_seed(0)
    q = torch.randn(2, 8, 64, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(2, 2, 96, 128, device="cuda").to(torch.bfloat16)
    v = torch.randn(2, 2, 96, 128, device="cuda").to(torch.bfloat16)
    for off in (-1, 32):
        torch.testing.assert_close(attn_prefill(q, k, v, causal_offset=off).float(),
                                   reference_attention(q, k, v, causal_offset=off).float(), atol=3e-2, rtol=3e-2)
    qd = q[:, :, :1]
    torch.testing.assert_close(attn_decode(qd, k, v, causal_offset=50).float(),
                               reference_attention(qd, k, v, causal_offset=50).float(), atol=3e-2, rtol=3e-2)
    kc = k.transpose(1, 2).reshape(2 * 6, 16, 2, 128).contiguous()  # 16-slot pages, reference layout
    vc = v.transpose(1, 2).reshape(2 * 6, 16, 2, 128).contiguous()
    table = torch.arange(12, device="cuda").view(2, 6)
    torch.testing.assert_close(attn_paged_decode(qd, table, kc, vc, 16, 96).float(),
                               reference_attention(qd, k, v).float(), atol=3e-2, rtol=3e-2)


def test_paged_decode_ignores_keys_beyond_the_table():
    """Lengths past the page table's capacity read no table entry past the row
    and no page outside the cache: those keys are skipped."""
    from astrai_b200.ops._ext import native

    C = native()
    kc, vc = _rand_cache(3, 2, 16, seed=5)
    table = torch.tensor([[2], [0]], dtype=torch.int32, device="cuda")  # one 16-slot page per row
    lens = torch.tensor([40, 16], dtype=torch.int32, device="cuda")     # row 0 claims 40 keys
    q = torch.randn(2, 4 * 128, device="cuda").to(torch.bfloat16)
    out = torch.empty_like(q)
    ws = torch.empty(2 * 4 * 3 * 130, device="cuda", dtype=torch.float32)
    C.paged_decode(q, kc, vc, table, lens, out, 4, 1 / math.sqrt(128), 3, ws)
    ref = torch.empty_like(q)
    C.paged_decode(q, kc, vc, table, torch.tensor([16, 16], dtype=torch.int32, device="cuda"), ref, 4,
                   1 / math.sqrt(128), 3, ws)
    torch.testing.assert_close(out.float(), ref.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("page", [16, 128])
def test_paged_decode_unwritten_slots_hold_nan(page):
    """Cache slots past a row's length (and whole unused pages) may hold anything, NaN included:
    the tensor-core kernel zeroes the V rows of those keys before the P V product, so NaN never
    reaches the output."""
    from astrai_b200.ops._ext import native

    C = native()
    torch.manual_seed(3)
    Hkv, G, D, B = 2, 8, 128, 3
    Hq = G * Hkv
    lens = [100, 300, 129]
    max_pages = max(-(-L // page) for L in lens)
    n_pages = B * max_pages
    kc, vc = _rand_cache(n_pages, Hkv, page, seed=9, D=D)
    table = torch.arange(n_pages, dtype=torch.int32, device="cuda").view(B, max_pages)
    kr, vr = _gather_ref(kc, vc, table, torch.tensor(lens, dtype=torch.int32, device="cuda"), max(lens))
    for b, L in enumerate(lens):  # poison every slot past the row's length
        for t in range(L, max_pages * page):
            pg = int(table[b, t // page])
            kc[pg, :, t % page] = float("nan")
            vc[pg, :, t % page] = float("nan")
    ln = torch.tensor(lens, dtype=torch.int32, device="cuda")
    q = torch.randn(B, Hq * D, device="cuda").to(torch.bfloat16)
    scale = 1 / math.sqrt(D)
    for splits in (1, 3):
        out = torch.empty(B, Hq * D, device="cuda", dtype=torch.bfloat16)
        ws = torch.empty(B * Hq * splits * (D + 2), device="cuda", dtype=torch.float32)
        C.paged_decode(q, kc, vc, table, ln, out, Hq, scale, splits, ws)
        assert torch.isfinite(out.float()).all()
        for b, L in enumerate(lens):
            qb = q[b].view(Hq, D).float()
            kb = kr[b, :L].repeat_interleave(G, dim=1)
            vb = vr[b, :L].repeat_interleave(G, dim=1)
            o = torch.einsum("hl,lhd->hd", torch.softmax(torch.einsum("hd,lhd->hl", qb, kb) * scale, -1), vb)
            torch.testing.assert_close(out[b].view(Hq, D).float(), o, atol=2e-2, rtol=2e-2)
