"""Flash-attention forward with two query tiles per CTA (flash_fwd_pair_kernel) against fp32 PyTorch.

Covers both pairings (two GQA heads at the same rows when Hq/Hkv is even, two row blocks of one head
otherwise), head_dim 64 and 128, partial tiles, queries that are the last Sq of Sk positions, no
causal mask, segment ids, and the one-tile kernel at the training shape. Output rows are written into
a wider canary-filled buffer so stray stores show up.
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
    assert native().read_error() == 0, "a kernel's bounded wait expired"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def run_pair(q, k, v, causal, seg=None):
    """q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] -> (o [B,Sq,Hq,D], lse [B,Hq,Sq]); o lives in a canary buffer."""
    from astrai_b200.ops._ext import native

    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    q2 = q.reshape(B * Sq, Hq * D).contiguous()
    kv = torch.cat([k.reshape(B * Sk, Hkv * D), v.reshape(B * Sk, Hkv * D)], 1).contiguous()
    canary = 77.0
    obuf = torch.full((B * Sq, Hq * D + 64), canary, device="cuda", dtype=torch.bfloat16)
    o = obuf[:, : Hq * D]
    lse = torch.empty(B, Hq, Sq, device="cuda", dtype=torch.float32)
    native().flash_fwd2(q2, 0, kv, 0, kv, Hkv * D, o, lse, B, Sq, Sk, Hq, Hkv, D, 1.0 / math.sqrt(D), causal, seg)
    torch.cuda.synchronize()
    assert (obuf[:, Hq * D:] == canary).all(), "stores past the output columns"
    return o.reshape(B, Sq, Hq, D), lse


def reference(q, k, v, causal, seg=None):
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    rep = Hq // Hkv
    qf = q.float().transpose(1, 2)
    kf = k.float().repeat_interleave(rep, 2).transpose(1, 2)
    vf = v.float().repeat_interleave(rep, 2).transpose(1, 2)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    mask = torch.ones(Sq, Sk, dtype=torch.bool, device=q.device)
    if causal:
        mask = torch.tril(mask, diagonal=Sk - Sq)
    mask = mask[None, None].expand(B, 1, Sq, Sk)
    if seg is not None:
        mask = mask & (seg[:, Sk - Sq:][:, None, :, None] == seg[:, None, None, :])
    s = s.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1).nan_to_num(0.0) @ vf
    return o.transpose(1, 2), lse


CASES = [  # B, Sq, Sk, Hq, Hkv, causal
    (1, 128, 128, 2, 1, True),     # pair heads, one block
    (2, 256, 256, 4, 2, True),     # pair heads
    (1, 300, 300, 4, 4, True),     # row pairs (G = 1), partial last tile, odd block count
    (1, 200, 200, 3, 1, True),     # row pairs (G = 3)
    (2, 384, 384, 8, 2, False),    # no mask
    (1, 1000, 1000, 8, 2, True),   # several key blocks, lazy rescales
    (2, 100, 612, 4, 2, True),     # queries are the last 100 of 612 positions
    (1, 1, 257, 4, 1, True),       # a single decode-like query row
]


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Sq,Sk,Hq,Hkv,causal", CASES)
def test_pair_forward_matches_fp32(D, B, Sq, Sk, Hq, Hkv, causal):
    torch.manual_seed(B * 131 + Sq + Sk + Hq + D)
    q = torch.randn(B, Sq, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, Sk, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, Sk, Hkv, D, device="cuda", dtype=torch.bfloat16)
    o, lse = run_pair(q, k, v, causal)
    of, lsef = reference(q, k, v, causal)
    assert rel_err(o, of) < 2e-2
    assert torch.allclose(lse, lsef, atol=2e-2, rtol=1e-3)


@pytest.mark.parametrize("D", [64, 128])
def test_pair_forward_segments(D):
    torch.manual_seed(12)
    B, S, Hq, Hkv = 2, 384, 4, 2
    seg = torch.zeros(B, S, dtype=torch.int32, device="cuda")
    seg[0, 100:] = 1
    seg[1, 37:180] = 1
    seg[1, 180:] = 2
    q = torch.randn(B, S, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    o, _ = run_pair(q, k, v, True, seg)
    of, _ = reference(q, k, v, True, seg)
    assert rel_err(o, of) < 2e-2


def test_pair_forward_large_scores_rescale():
    """Scores that grow along the keys force repeated rescales of the O accumulator."""
    torch.manual_seed(13)
    B, S, Hq, Hkv, D = 1, 1024, 2, 1, 128
    q = torch.randn(B, S, Hq, D, device="cuda", dtype=torch.bfloat16)
    ramp = torch.linspace(0.2, 6.0, S, device="cuda")[None, :, None, None]
    k = (torch.randn(B, S, Hkv, D, device="cuda") * ramp).to(torch.bfloat16)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    o, lse = run_pair(q, k, v, True)
    of, lsef = reference(q, k, v, True)
    assert rel_err(o, of) < 2e-2
    assert torch.allclose(lse, lsef, atol=5e-2, rtol=1e-3)


def test_pair_and_one_tile_kernels_agree_at_training_shape():
    from astrai_b200.ops._ext import native

    torch.manual_seed(14)
    B, S, Hq, Hkv, D = 2, 2048, 16, 4, 128
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
    outs = []
    for fn in ("flash_fwd", "flash_fwd2"):
        o = torch.empty(B * S, Hq * D, device="cuda", dtype=torch.bfloat16)
        lse = torch.empty(B, Hq, S, device="cuda", dtype=torch.float32)
        args = (qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, lse, B, S, S, Hq, Hkv)
        if fn == "flash_fwd2":
            native().flash_fwd2(*args, D, 1.0 / math.sqrt(D), True, None)
        else:
            native().flash_fwd(*args, 1.0 / math.sqrt(D), True, None)
        outs.append((o, lse))
    assert rel_err(outs[1][0], outs[0][0]) < 1e-2
    assert torch.allclose(outs[1][1], outs[0][1], atol=1e-2)


def test_inference_attention_head_dim_64_uses_kernel():
    """``ops.attention.attention`` without autograd runs the pair kernel for head_dim 64."""
    from astrai_b200.ops.attention import attention

    torch.manual_seed(15)
    B, S, Hq, Hkv, D = 2, 192, 6, 2, 64
    q = torch.randn(B, S, Hq, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(B, S, Hkv, D, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        o = attention(q, k, v, causal=True)
    of, _ = reference(q, k, v, True)
    assert rel_err(o, of) < 2e-2
