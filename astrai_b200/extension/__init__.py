"""Standalone attention ops with the reference extension's interface.

API parity with astrai/extension (``__init__.py``, ``loader.py:14-36``,
``ops.py:170-298``): ``attn_prefill``, ``attn_decode``, ``attn_paged_decode``,
``attention`` (dispatch on query length), ``is_available``, ``KERNEL_NAMES``.

Interface, as in the reference:
  layout        "bhld" (default) or "blhd"
  causal_offset -1 = not causal; >= 0 = absolute position of the first query
  mask          bool [batch, kv_len] or [batch, q_len, kv_len], True = keep
  scale         0.0 = 1/sqrt(head_dim)

Execution: bf16 CUDA inputs with head_dim 128 run on this framework's
sm_100a kernels (flash attention for prefill when the causal offset is the
bottom-right one or absent, the paged split-KV decode kernel for decode,
reading contiguous K/V as one page per sequence). An explicit mask, another
causal offset, head dim or dtype takes the dense fp32 path of
:func:`reference_attention`, which is also the CPU implementation.
``attn_paged_decode`` accepts the reference's cache layout
``[n_pages, page_size, n_kv_heads, head_dim]`` (``cache_layout="pshd"``,
default) or this framework's ``[n_pages, n_kv_heads, page_size, head_dim]``
(``"phsd"``, no copy).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

KERNEL_NAMES = ["attn_decode", "attn_prefill", "attn_paged_decode"]


def is_available(name: str) -> bool:
    """True when the compiled sm_100a kernels behind ``name`` are loadable here."""
    if name not in KERNEL_NAMES or not torch.cuda.is_available():
        return False
    try:
        from astrai_b200.ops._ext import native

        native()
        return True
    except (ImportError, RuntimeError):
        return False


def _li(layout) -> int:
    if layout in (0, "bhld"):
        return 0
    if layout in (1, "blhd"):
        return 1
    raise ValueError(f"layout must be 'bhld' or 'blhd', got {layout!r}")


def _bhld(t: torch.Tensor, li: int) -> torch.Tensor:
    return t if li == 0 else t.transpose(1, 2)


def reference_attention(q, k, v, mask=None, causal_offset: int = -1, scale: float = 0.0, layout="bhld"):
    """Dense fp32 attention with GQA head sharing (any device)."""
    li = _li(layout)
    qb, kb, vb = (_bhld(t, li).float() for t in (q, k, v))
    B, Hq, Lq, D = qb.shape
    Hkv, Lk = kb.shape[1], kb.shape[2]
    rep = Hq // Hkv
    if rep > 1:
        kb, vb = kb.repeat_interleave(rep, 1), vb.repeat_interleave(rep, 1)
    sc = scale if scale > 0 else 1.0 / math.sqrt(D)
    s = (qb @ kb.transpose(-1, -2)) * sc
    keep = torch.ones(B, 1, Lq, Lk, dtype=torch.bool, device=q.device)
    if causal_offset >= 0:
        qpos = causal_offset + torch.arange(Lq, device=q.device)
        keep = keep & (torch.arange(Lk, device=q.device)[None, :] <= qpos[:, None])[None, None]
    if mask is not None:
        m = mask.bool().to(q.device)
        keep = keep & (m[:, None, None, :] if m.dim() == 2 else m[:, None])
    s = s.masked_fill(~keep, float("-inf"))
    o = torch.softmax(s, -1).nan_to_num(0.0) @ vb
    o = o.to(q.dtype)
    return o if li == 0 else o.transpose(1, 2)


def _native_ok(*ts) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 and t.shape[-1] == 128 for t in ts)


def attn_prefill(q, k, v, mask=None, causal_offset: int = -1, scale: float = 0.0, layout="bhld"):
    li = _li(layout)
    qb, kb, vb = (_bhld(t, li) for t in (q, k, v))
    Lq, Lk = qb.shape[2], kb.shape[2]
    bottom_right = causal_offset == Lk - Lq
    if mask is None and (causal_offset < 0 or bottom_right) and (scale <= 0 or abs(scale - 128 ** -0.5) < 1e-9) \
            and _native_ok(q, k, v):
        from astrai_b200.ops.attention import attention as flash

        o = flash(qb.transpose(1, 2), kb.transpose(1, 2), vb.transpose(1, 2), causal=causal_offset >= 0)
        o = o.transpose(1, 2)  # [B, Hq, Lq, D]
        return o if li == 0 else o.transpose(1, 2)
    return reference_attention(q, k, v, mask, causal_offset, scale, layout)


def _decode_pages(qb: torch.Tensor, kc, vc, table, lens, scale: float) -> torch.Tensor:
    """qb [B, Hq, 1, 128]; kc / vc [n_pages, Hkv, page, 128] -> [B, Hq, 1, 128]."""
    from astrai_b200.ops._ext import native

    C = native()
    B, Hq = qb.shape[0], qb.shape[1]
    q2 = qb.reshape(B, Hq * 128).contiguous()
    out = torch.empty_like(q2)
    splits = int(C.decode_splits(B, kc.shape[1], table.shape[1] * kc.shape[2], q2.device.index or 0))
    ws = torch.empty(B * Hq * splits * 130, device=q2.device, dtype=torch.float32) if splits > 1 else None
    C.paged_decode(q2, kc, vc, table, lens, out, Hq, scale if scale > 0 else 128 ** -0.5, splits, ws)
    return out.view(B, Hq, 1, 128)


def attn_decode(q, k, v, mask=None, causal_offset: int = -1, scale: float = 0.0, layout="bhld"):
    li = _li(layout)
    qb, kb, vb = (_bhld(t, li) for t in (q, k, v))
    B, Lk = qb.shape[0], kb.shape[2]
    if mask is None and qb.shape[2] == 1 and _native_ok(q, k, v):
        n = Lk if causal_offset < 0 else min(Lk, causal_offset + 1)
        kc, vc = kb.contiguous(), vb.contiguous()  # one "page" of Lk keys per sequence
        table = torch.arange(B, device=q.device, dtype=torch.int32).view(B, 1)
        lens = torch.full((B,), n, device=q.device, dtype=torch.int32)
        o = _decode_pages(qb, kc, vc, table, lens, scale)
        return o if li == 0 else o.transpose(1, 2)
    return reference_attention(q, k, v, mask, causal_offset, scale, layout)


def attn_paged_decode(q, page_table, k_cache, v_cache, page_size: int, kv_len: int, mask=None,
                      causal_offset: int = -1, scale: float = 0.0, layout="bhld", cache_layout: str = "pshd"):
    li = _li(layout)
    qb = _bhld(q, li)
    if cache_layout not in ("pshd", "phsd"):
        raise ValueError("cache_layout must be 'pshd' or 'phsd'")
    kc = k_cache if cache_layout == "phsd" else k_cache.permute(0, 2, 1, 3)
    vc = v_cache if cache_layout == "phsd" else v_cache.permute(0, 2, 1, 3)
    if kc.shape[2] != page_size:
        raise ValueError(f"k_cache page_size mismatch: {kc.shape[2]} vs {page_size}")
    B = qb.shape[0]
    n = kv_len if causal_offset < 0 else min(kv_len, causal_offset + 1)
    if mask is None and qb.shape[2] == 1 and _native_ok(q, kc, vc):
        lens = torch.full((B,), n, device=q.device, dtype=torch.int32)
        o = _decode_pages(qb, kc.contiguous(), vc.contiguous(), page_table.to(torch.int32).contiguous(), lens, scale)
        return o if li == 0 else o.transpose(1, 2)
    pos = torch.arange(kv_len, device=q.device)
    pages = page_table.long()[:, pos // page_size].clamp(min=0)
    k = kc[pages, :, pos % page_size].permute(0, 2, 1, 3)  # [B, Hkv, L, D]
    v = vc[pages, :, pos % page_size].permute(0, 2, 1, 3)
    return reference_attention(qb, k, v, mask, causal_offset, scale, "bhld") if li == 0 else \
        reference_attention(qb, k, v, mask, causal_offset, scale, "bhld").transpose(1, 2)


def attention(q, k, v, mask=None, causal_offset: int = -1, scale: float = 0.0, layout="bhld"):
    """Decode when the query length is 1, prefill otherwise (2-D / 3-D inputs allowed)."""
    li = _li(layout)
    if q.ndim not in (2, 3, 4) or k.ndim != q.ndim or v.ndim != q.ndim:
        raise ValueError(f"q, k, and v must all have the same rank in {{2, 3, 4}}, got {q.ndim}D, {k.ndim}D, {v.ndim}D")
    if k.shape != v.shape:
        raise ValueError(f"k and v must have the same shape, got {k.shape} and {v.shape}")
    nd = q.ndim
    hd = 1 if li == 0 else 2
    if nd == 2:
        q, k, v = (t.unsqueeze(0).unsqueeze(hd) for t in (q, k, v))
    elif nd == 3:
        q, k, v = (t.unsqueeze(hd) for t in (q, k, v))
    lq = q.shape[2 if li == 0 else 1]
    fn = attn_decode if lq == 1 else attn_prefill
    out = fn(q, k, v, mask, causal_offset, scale, layout)
    if nd == 2:
        return out.squeeze(0).squeeze(0 if li == 0 else 1)
    if nd == 3:
        return out.squeeze(hd)
    return out


__all__ = ["KERNEL_NAMES", "attention", "attn_decode", "attn_paged_decode", "attn_prefill", "is_available",
           "reference_attention"]
