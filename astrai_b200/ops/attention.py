"""Attention ops.

* :func:`attention_qkv` - the training hot path. Takes the fused QKV
  projection output ``[B*S, (Hq + 2*Hkv) * D]``, applies interleaved RoPE in
  place to the q and k heads and runs the tcgen05 flash-attention kernels
  (causal, GQA without repeating K/V, optional document segments). Returns
  ``[B*S, Hq*D]``, the layout the o-projection consumes.
* :func:`attention` - generic ``[B, S, H, D]`` q/k/v (MLA, encoder, prefill
  with a KV cache): copies into row buffers and runs the same kernels.

Semantics match the reference's SDPA call (astrai/model/components/attention.py:96-101):
softmax scale ``1/sqrt(D)``, causal masking aligned to the end of the key
sequence (queries are the last ``Sq`` positions), GQA head ``h`` reads K/V head
``h // (Hq // Hkv)``. Document masks (SFT packing, strategy.py:79-92) and
key-padding masks (DPO/GRPO) are passed as int32 segment ids: query q sees key
k only if ``seg[q] == seg[k]`` (padding keys get unique negative ids).

On CUDA the forward runs ``flash_fwd_pair_kernel`` (two query tiles per CTA, P kept in tensor
memory; head_dim 64 or 128); ``ASTRAI_FLASH_FWD_PAIR=0`` selects the one-tile kernel
(head_dim 128 only). The backward kernel covers head_dim 128. CPU tensors and other head sizes
use the PyTorch reference math below.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from astrai_b200.ops._ext import native
from astrai_b200.ops.rope import apply_rope_reference, rope_inplace

HEAD_DIM = 128
FWD_HEAD_DIMS = (64, 128)
PAIR_FWD = __import__("os").environ.get("ASTRAI_FLASH_FWD_PAIR", "1") != "0"


def flash_forward(q, q_col0, k, k_col0, v, v_col0, o, lse, B, Sq, Sk, Hq, Hkv, D, scale, causal, seg):
    """Forward kernel on row buffers (head ``h`` of q at columns ``q_col0 + h*D``, same for k/v)."""
    C = native()
    if PAIR_FWD:
        C.flash_fwd2(q, q_col0, k, k_col0, v, v_col0, o, lse, B, Sq, Sk, Hq, Hkv, D, scale, causal, seg)
    else:
        assert D == HEAD_DIM, "the one-tile forward kernel supports head_dim 128 only"
        C.flash_fwd(q, q_col0, k, k_col0, v, v_col0, o, lse, B, Sq, Sk, Hq, Hkv, scale, causal, seg)


# ----------------------------------------------------------------------------- reference math
def attention_reference(q, k, v, causal=True, seg=None, scale=None):
    """q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] -> [B,Sq,Hq,D] (fp32 math, input dtype out)."""
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    rep = Hq // Hkv
    kk = k.repeat_interleave(rep, dim=2) if rep > 1 else k
    vv = v.repeat_interleave(rep, dim=2) if rep > 1 else v
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, kk, vv))
    mask = torch.ones(Sq, Sk, dtype=torch.bool, device=q.device)
    if causal:
        mask = torch.tril(mask, diagonal=Sk - Sq)
    mask = mask[None, None].expand(B, 1, Sq, Sk)
    if seg is not None:
        sq = seg[:, Sk - Sq:]
        mask = mask & (sq[:, None, :, None] == seg[:, None, None, :])
    s = (qf @ kf.transpose(-1, -2)) * (scale if scale is not None else 1.0 / math.sqrt(D))
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    o = p @ vf
    return o.transpose(1, 2).to(q.dtype)


def _sdpa(q, k, v, causal, seg, scale=None):
    """PyTorch path (CPU / unsupported head sizes)."""
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    if seg is None and (not causal or Sq == Sk):
        rep = Hq // Hkv
        kk = k.repeat_interleave(rep, dim=2) if rep > 1 else k
        vv = v.repeat_interleave(rep, dim=2) if rep > 1 else v
        o = F.scaled_dot_product_attention(q.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2),
                                           is_causal=causal, scale=scale)
        return o.transpose(1, 2)
    return attention_reference(q, k, v, causal, seg, scale)


# ----------------------------------------------------------------------------- fused training path
class _AttnQKVFn(torch.autograd.Function):
    """``rotated``: q/k already carry RoPE (applied in the QKV projection epilogue), so neither the
    forward rotation nor the backward inverse rotation happens here."""

    @staticmethod
    def forward(ctx, qkv, table, positions, seg, B, S, Hq, Hkv, causal, rotated=False):
        D = HEAD_DIM
        C = native()
        if not rotated:
            rope_inplace(qkv, 0, Hq + Hkv, D, table, positions, S)  # q and k heads are adjacent
        o = torch.empty((B * S, Hq * D), device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty((B, Hq, S), device=qkv.device, dtype=torch.float32)
        flash_forward(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, lse, B, S, S, Hq, Hkv, D, 1.0 / math.sqrt(D),
                      causal, seg)
        ctx.save_for_backward(qkv, o, lse, table, positions, seg)
        ctx.dims = (B, S, Hq, Hkv, causal)
        ctx.rotated = rotated
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse, table, positions, seg = ctx.saved_tensors
        B, S, Hq, Hkv, causal = ctx.dims
        D = HEAD_DIM
        C = native()
        do = do.contiguous()
        dqkv = torch.empty_like(qkv)
        dq_acc = torch.empty((B * S, Hq * D), device=qkv.device, dtype=torch.float32)  # zeroed by the kernel
        delta = torch.empty(2 * B * Hq * ((S + 63) // 64 * 64), device=qkv.device, dtype=torch.float32)
        C.flash_bwd(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, do, lse, delta, dq_acc, dqkv, 0, dqkv, Hq * D,
                    dqkv, (Hq + Hkv) * D, B, S, S, Hq, Hkv, 1.0 / math.sqrt(D), causal, seg)
        if not ctx.rotated:
            rope_inplace(dqkv, 0, Hq + Hkv, D, table, positions, S, inverse=True)
        return dqkv, None, None, None, None, None, None, None, None, None


def attention_qkv(qkv: torch.Tensor, B: int, S: int, Hq: int, Hkv: int, table: torch.Tensor,
                  positions: Optional[torch.Tensor] = None, causal: bool = True,
                  seg: Optional[torch.Tensor] = None, rotated: bool = False) -> torch.Tensor:
    """RoPE + attention on a fused QKV buffer ``[B*S, (Hq+2Hkv)*D]``.

    ``table`` is the fp32 (cos, sin) table ``[max_pos, D/2, 2]`` on the same
    device; ``positions`` int [B, S] (None -> 0..S-1 per sequence).
    On CUDA the buffer is rotated in place, unless ``rotated`` (RoPE already applied by the
    projection epilogue, see :func:`astrai_b200.ops.gemm.packed_linear_rope`).
    """
    D = qkv.shape[-1] // (Hq + 2 * Hkv)
    if qkv.is_cuda and qkv.dtype == torch.bfloat16 and D == HEAD_DIM:
        pos = positions.reshape(-1).to(torch.int32).contiguous() if positions is not None else None
        sg = seg.to(torch.int32).contiguous() if seg is not None else None
        return _AttnQKVFn.apply(qkv, table, pos, sg, B, S, Hq, Hkv, causal, rotated)
    if (qkv.is_cuda and qkv.dtype == torch.bfloat16 and D in FWD_HEAD_DIMS and PAIR_FWD
            and not (torch.is_grad_enabled() and qkv.requires_grad) and qkv.is_contiguous()):
        # forward only (prefill, evaluation) at another head size: RoPE in place on the fresh projection
        # output, then the forward kernel (the backward kernel covers head_dim 128 only)
        pos = positions.reshape(-1).to(torch.int32).contiguous() if positions is not None else None
        sg = seg.to(torch.int32).contiguous() if seg is not None else None
        if not rotated:
            rope_inplace(qkv, 0, Hq + Hkv, D, table, pos, S)
        o = torch.empty((B * S, Hq * D), device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty((B, Hq, S), device=qkv.device, dtype=torch.float32)
        flash_forward(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, lse, B, S, S, Hq, Hkv, D, 1.0 / math.sqrt(D),
                      causal, sg)
        return o
    q, k, v = qkv.view(B, S, Hq + 2 * Hkv, D).split([Hq, Hkv, Hkv], dim=2)
    if not rotated:
        if positions is None:
            cs = table[:S].unsqueeze(0).expand(B, -1, -1, -1)
        else:
            cs = table[positions]
        q = apply_rope_reference(q, cs)
        k = apply_rope_reference(k, cs)
    return _sdpa(q, k, v, causal, seg).reshape(B * S, Hq * D)


# ----------------------------------------------------------------------------- generic path
class _AttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, seg, causal):
        B, Sq, Hq, D = q.shape
        Sk, Hkv = k.shape[1], k.shape[2]
        C = native()
        q2 = q.reshape(B * Sq, Hq * D).contiguous()
        k2 = k.reshape(B * Sk, Hkv * D).contiguous()
        v2 = v.reshape(B * Sk, Hkv * D).contiguous()
        o = torch.empty((B * Sq, Hq * D), device=q.device, dtype=torch.bfloat16)
        lse = torch.empty((B, Hq, Sq), device=q.device, dtype=torch.float32)
        flash_forward(q2, 0, k2, 0, v2, 0, o, lse, B, Sq, Sk, Hq, Hkv, D, 1.0 / math.sqrt(D), causal, seg)
        ctx.save_for_backward(q2, k2, v2, o, lse, seg)
        ctx.dims = (B, Sq, Sk, Hq, Hkv, causal)
        return o.view(B, Sq, Hq, D)

    @staticmethod
    def backward(ctx, do):
        q2, k2, v2, o, lse, seg = ctx.saved_tensors
        B, Sq, Sk, Hq, Hkv, causal = ctx.dims
        D = HEAD_DIM
        C = native()
        do2 = do.reshape(B * Sq, Hq * D).contiguous()
        dq = torch.empty_like(q2)
        dkv = torch.empty((B * Sk, 2 * Hkv * D), device=q2.device, dtype=torch.bfloat16)
        dq_acc = torch.empty((B * Sq, Hq * D), device=q2.device, dtype=torch.float32)  # zeroed by the kernel
        delta = torch.empty(2 * B * Hq * ((Sq + 63) // 64 * 64), device=q2.device, dtype=torch.float32)
        C.flash_bwd(q2, 0, k2, 0, v2, 0, o, do2, lse, delta, dq_acc, dq, 0, dkv, 0, dkv, Hkv * D, B, Sq, Sk, Hq, Hkv,
                    1.0 / math.sqrt(D), causal, seg)
        dk = dkv[:, : Hkv * D].reshape(B, Sk, Hkv, D)
        dv = dkv[:, Hkv * D:].reshape(B, Sk, Hkv, D)
        return dq.view(B, Sq, Hq, D), dk, dv, None, None


def _forward_only(q, k, v, seg, causal):
    """Kernel forward without autograd state (inference, or head sizes the backward kernel lacks)."""
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    q2 = q.reshape(B * Sq, Hq * D).contiguous()
    k2 = k.reshape(B * Sk, Hkv * D).contiguous()
    v2 = v.reshape(B * Sk, Hkv * D).contiguous()
    o = torch.empty((B * Sq, Hq * D), device=q.device, dtype=torch.bfloat16)
    lse = torch.empty((B, Hq, Sq), device=q.device, dtype=torch.float32)
    flash_forward(q2, 0, k2, 0, v2, 0, o, lse, B, Sq, Sk, Hq, Hkv, D, 1.0 / math.sqrt(D), causal, seg)
    return o.view(B, Sq, Hq, D)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              seg: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] -> [B,Sq,Hq,D]."""
    D = q.shape[-1]
    kernel_ok = q.is_cuda and q.dtype == torch.bfloat16 and k.shape[-1] == D and v.shape[-1] == D
    if kernel_ok and D == HEAD_DIM:
        sg = seg.to(torch.int32).contiguous() if seg is not None else None
        return _AttnFn.apply(q, k, v, sg, causal)
    grad = torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v))
    if kernel_ok and PAIR_FWD and D in FWD_HEAD_DIMS and not grad:
        sg = seg.to(torch.int32).contiguous() if seg is not None else None
        return _forward_only(q, k, v, sg, causal)
    return _sdpa(q, k, v, causal, seg)


def bench_attention(time_fn, peaks):
    """Device-timed flash attention fwd / fwd+bwd at the 1.1B training shape."""
    import json

    hbm, tf, src = peaks()
    B, S, Hq, Hkv, D = 4, 2048, 16, 4, 128
    qkv = torch.randn(B * S, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
    from astrai_b200.ops.rope import rope_table

    table = rope_table(D, S, 1e6, device="cuda")
    C = native()
    o = torch.empty(B * S, Hq * D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, Hq, S, device="cuda", dtype=torch.float32)
    scale = 1.0 / math.sqrt(D)
    fwd1 = lambda: C.flash_fwd(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, lse, B, S, S, Hq, Hkv, scale, True, None)
    fwd = lambda: C.flash_fwd2(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, lse, B, S, S, Hq, Hkv, D, scale, True,
                               None)
    ms1 = time_fn(fwd1)
    ms = time_fn(fwd)
    flops = 4.0 * B * Hq * S * S * D / 2  # causal
    q = qkv[:, : Hq * D].view(B, S, Hq, D).transpose(1, 2)
    kk = qkv[:, Hq * D: (Hq + Hkv) * D].view(B, S, Hkv, D).transpose(1, 2)
    vv = qkv[:, (Hq + Hkv) * D:].view(B, S, Hkv, D).transpose(1, 2)
    ref = lambda: F.scaled_dot_product_attention(q, kk, vv, is_causal=True, enable_gqa=True)
    ms_ref = time_fn(ref)
    print(json.dumps({"kernel": "flash_fwd_pair", "B": B, "S": S, "Hq": Hq, "Hkv": Hkv, "ms": round(ms, 4),
                      "one_tile_kernel_ms": round(ms1, 4),
                      "tflops": round(flops / ms / 1e9, 1), "frac_of_peak": round(flops / ms / 1e9 / tf, 3),
                      "peak_src": src, "sdpa_ms": round(ms_ref, 4), "sdpa_tflops": round(flops / ms_ref / 1e9, 1)}))
    do = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(B * S, Hq * D, device="cuda", dtype=torch.float32)
    delta = torch.empty(2 * B * Hq * S, device="cuda", dtype=torch.float32)

    def bwd():
        C.flash_bwd(qkv, 0, qkv, Hq * D, qkv, (Hq + Hkv) * D, o, do, lse, delta, dq_acc, dqkv, 0, dqkv, Hq * D, dqkv,
                    (Hq + Hkv) * D, B, S, S, Hq, Hkv, scale, True, None)

    ms_b = time_fn(bwd)
    qr, kr, vr = (t.detach().clone().requires_grad_() for t in (q, kk, vv))
    out = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True, enable_gqa=True)
    g = torch.randn_like(out)
    ms_rb = time_fn(lambda: torch.autograd.grad(out, (qr, kr, vr), g, retain_graph=True))
    print(json.dumps({"kernel": "flash_bwd", "ms": round(ms_b, 4), "tflops": round(2.5 * flops / ms_b / 1e9, 1),
                      "frac_of_peak": round(2.5 * flops / ms_b / 1e9 / tf, 3), "sdpa_bwd_ms": round(ms_rb, 4),
                      "sdpa_bwd_tflops": round(2.5 * flops / ms_rb / 1e9, 1)}))
