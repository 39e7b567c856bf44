"""Whole-model numerics: the CUDA (bf16, native kernels) path against the CPU
fp32 oracle with identical weights, forward and backward, plus a few
optimizer steps of the fused Muon/AdamW against their torch references."""

import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(a, b):
    a, b = a.float().cpu(), b.float().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def tiny_cfg(**kw):
    from astrai_b200.config import AutoRegressiveLMConfig

    base = dict(vocab_size=512, hidden_size=256, num_hidden_layers=2, rms_norm_eps=1e-5, intermediate_size=512,
                tie_word_embeddings=False, max_position_embeddings=512, rope_theta=10000.0, num_attention_heads=2,
                num_key_value_heads=1)
    base.update(kw)
    return AutoRegressiveLMConfig(**base)


VARIANTS = {
    "gqa": {},
    "tied": dict(tie_word_embeddings=True),
    # the attention options of the reference's model config, on the kernel path (head_dim 128)
    "qk_norm_gated": dict(use_qk_norm=True, use_gated_attention=True),
    "mla": dict(attn_type="mla", num_attention_heads=2, num_key_value_heads=2, kv_lora_rank=64,
                qk_nope_head_dim=96, qk_rope_head_dim=32),
    "mla_qk_norm_gated": dict(attn_type="mla", num_attention_heads=2, num_key_value_heads=1, kv_lora_rank=64,
                              qk_nope_head_dim=96, qk_rope_head_dim=32, use_qk_norm=True, use_gated_attention=True),
}


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_lm_forward_backward_matches_cpu(variant):
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.loss import cross_entropy

    torch.manual_seed(0)
    cpu = AutoRegressiveLM(tiny_cfg(**VARIANTS[variant])).float()
    gpu = copy.deepcopy(cpu).cuda().to(torch.bfloat16)
    # compare against the bf16-rounded weights so only compute precision differs
    cpu.load_state_dict({k: v.to(torch.bfloat16).float() for k, v in cpu.state_dict().items()})
    ids = torch.randint(0, 512, (2, 200))
    tgt = torch.randint(0, 512, (2, 200))
    lc = cross_entropy(cpu(ids)["logits"], tgt, label_smoothing=0.05)
    lc.backward()
    lg = cross_entropy(gpu(ids.cuda())["logits"], tgt.cuda(), label_smoothing=0.05)
    lg.backward()
    torch.cuda.synchronize()
    assert native().read_error() == 0
    assert abs(lc.item() - lg.item()) < 2e-2
    gc = dict(cpu.named_parameters())
    for n, p in gpu.named_parameters():
        assert rel(p.grad, gc[n].grad) < 6e-2, n


@pytest.mark.parametrize("chunk_bytes", [None, 1])
def test_fused_optimizers_match_torch(chunk_bytes, monkeypatch):
    """chunk_bytes=1: every batched Newton-Schulz chain holds one matrix (the chunked path)."""
    import astrai_b200.optim.fused as fused
    from astrai_b200.optim import FusedAdamW, Muon, clip_grad_norm_, newton_schulz_reference

    if chunk_bytes is not None:
        monkeypatch.setattr(fused, "_NS_CHUNK_BYTES", chunk_bytes)
    torch.manual_seed(1)
    # vector normalize / apply paths (multiples of 64, 8-element rows) and the element-wise ones
    shapes = [(256, 512), (512, 256), (256, 512), (128, 128), (96, 200), (200, 96)]
    ps = [torch.randn(s, device="cuda").to(torch.bfloat16) for s in shapes]
    ref = [p.clone() for p in ps]
    grads = [torch.randn_like(p) for p in ps]
    P = [torch.nn.Parameter(p) for p in ps]
    for p, g in zip(P, grads):
        p.grad = g.clone()
    opt = Muon(P, lr=0.02, weight_decay=0.1, adjust_lr_fn="match_rms_adamw")
    opt.step()
    for p0, g, p in zip(ref, grads, P):
        buf = 0.05 * g.float()  # first step: momentum buffer = (1 - mu) * g
        u = g.float() + 0.95 * (buf - g.float())
        upd = newton_schulz_reference(u, 5).float()
        adj = 0.02 * 0.2 * max(p0.shape) ** 0.5
        exp = p0.float() * (1 - 0.02 * 0.1) - adj * upd
        assert rel(p.data, exp) < 2e-2
    # AdamW + on-device clip coefficient
    w = torch.nn.Parameter(torch.randn(1003, device="cuda").to(torch.bfloat16))  # 16-byte loads + a 3-element tail
    w.grad = (torch.randn(1003, device="cuda") * 10).to(torch.bfloat16)
    wt = torch.nn.Parameter(w.detach().float().clone())
    wt.grad = w.grad.float().clone()
    n = clip_grad_norm_([w], 1.0)
    torch.nn.utils.clip_grad_norm_([wt], 1.0)
    FusedAdamW([w], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1).step()
    torch.optim.AdamW([wt], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1).step()
    assert rel(w.data, wt.data) < 1e-2
    assert abs(float(n) - float(torch.linalg.vector_norm(w.grad.float()))) < 1e-1 * float(n)


@pytest.mark.parametrize("heads,kv", [(4, 2), (6, 1)])
def test_forward_only_head_dim_64_matches_cpu(heads, kv):
    """head_dim 64 without gradients (prefill, evaluation): RoPE in place and the forward kernel on the
    fused QKV buffer, against the fp32 CPU oracle."""
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.ops._ext import native

    torch.manual_seed(1)
    cpu = AutoRegressiveLM(tiny_cfg(hidden_size=64 * heads, num_attention_heads=heads, num_key_value_heads=kv,
                                    intermediate_size=512)).float().eval()
    cpu.load_state_dict({k: v.to(torch.bfloat16).float() for k, v in cpu.state_dict().items()})
    gpu = copy.deepcopy(cpu).cuda().to(torch.bfloat16).eval()
    ids = torch.randint(0, 512, (2, 300))
    with torch.inference_mode():
        lg = gpu(ids.cuda())["logits"]
    torch.cuda.synchronize()
    assert native().read_error() == 0
    lc = cpu(ids)["logits"].detach()
    assert rel(lg, lc) < 2e-2
