"""Linear layers on the tcgen05 GEMM.

``linear(x, w, residual=None)`` computes ``x @ w.T (+ residual)`` with
``w`` stored ``[out, in]`` like the reference Linear
(astrai/model/components/linear.py:7-24). Forward, data-grad and weight-grad
all run on the same persistent sm_100a kernel; the three products only differ
in which operand is K-major and which is MN-major, so no transposed copies of
activations or weights are made. A residual passed in is added in the GEMM
epilogue (used for the o_proj / down projections of a pre-norm block).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from astrai_b200.ops._ext import native


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, *, a_mn: bool = False,
         b_mn: bool = False, c: Optional[torch.Tensor] = None, alpha: float = 1.0, beta: float = 0.0,
         out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """D = alpha * op(a) @ op(b)^T + beta * c on CUDA (bf16 inputs).

    a: [M, K] (a_mn False) or [K, M] (a_mn True); b: [N, K] or [K, N];
    3-D inputs are batched over dim 0.
    """
    batched = a.dim() == 3
    M = a.shape[-1] if a_mn else a.shape[-2]
    N = b.shape[-1] if b_mn else b.shape[-2]
    if out is None:
        shape = (a.shape[0], M, N) if batched else (M, N)
        out = torch.empty(shape, device=a.device, dtype=out_dtype)
    native().gemm(a, b, out, c, int(a_mn), int(b_mn), float(alpha), float(beta), 0)
    return out


def gemm_reference(a, b, *, a_mn=False, b_mn=False, c=None, alpha=1.0, beta=0.0):
    """fp32 oracle of :func:`gemm` (any device)."""
    A = a.float().transpose(-1, -2) if a_mn else a.float()
    B = b.float().transpose(-1, -2) if b_mn else b.float()
    d = alpha * (A @ B.transpose(-1, -2))
    if c is not None:
        d = d + beta * c.float()
    return d


def _as_rows(t: torch.Tensor) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1 or (t2.stride(0) * t2.element_size()) % 16:
        t2 = t2.contiguous()
    return t2


SKINNY_MAX_ROWS = 16
# False while torch ``fully_shard`` manages the parameters: its unsharded parameters live in buffers it
# frees and refills, so they must not be re-pointed into packed buffers (packed projections then
# concatenate their weights per call instead)
PACKING = True


def set_packing(enabled: bool) -> None:
    global PACKING
    PACKING = bool(enabled)

# SwiGLU / RoPE in GEMM epilogues (gemm_swiglu, gemm_rope): correct, but measured slower on B200 in
# the 1.1B training step (the 4 epilogue warps of a 128-row tile become the bottleneck once they
# carry the extra memory traffic, and the larger 256-row tiles cannot hold the registers), so the
# separate full-GPU kernels are the default; set ASTRAI_FUSED_EPILOGUES=1 to use the fused ones.
FUSED_EPILOGUES = __import__("os").environ.get("ASTRAI_FUSED_EPILOGUES", "0") == "1"
# The SwiGLU pair alone (ASTRAI_FUSED_SWIGLU=1): its GEMMs run on 256-row CTA-pair tiles, whose
# accumulators are double-buffered like the 128-row tiles', so the epilogue work overlaps the MMAs.
# Still measured slower in the 1.1B step on B200 (613 - 618 vs 586 - 590 ms per optimizer step, two
# runs each on one box), so it stays opt-in.
FUSED_SWIGLU = FUSED_EPILOGUES or __import__("os").environ.get("ASTRAI_FUSED_SWIGLU", "0") == "1"
# Without autograd (prefill, rollouts, evaluation) the SwiGLU GEMM stores only a = silu(g) * u, not
# h = (u, g): one GEMM replaces the packed up/gate GEMM, the h round trip and the SwiGLU kernel.
# ASTRAI_INFER_SWIGLU=0 keeps the separate kernels there.
INFER_SWIGLU = __import__("os").environ.get("ASTRAI_INFER_SWIGLU", "1") == "1"
# RoPE in the QKV projection's epilogue (the CTA-pair tiles rotate q and k before the store; the
# attention kernel then skips its own rotation, and the backward rotates the gradient back in place).
# Measured on B200: the reference benchmark's prefill forward 4.56 -> 4.21 ms; the 1.1B step is
# unchanged within run-to-run noise (547.3 vs 549.7 ms on one box). ASTRAI_FUSED_ROPE=0 keeps the
# separate in-place kernel.
FUSED_ROPE = FUSED_EPILOGUES or __import__("os").environ.get("ASTRAI_FUSED_ROPE", "1") == "1"


def _skinny(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """Decode-shaped products (<= 16 rows, no autograd): the skinny kernel that
    streams the weight once over the whole GPU. None when not applicable."""
    if torch.is_grad_enabled():
        return None
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[0] > SKINNY_MAX_ROWS or x2.shape[0] == 0:
        return None
    x2 = _as_rows(x2)
    out = torch.empty((x2.shape[0], w.shape[0]), device=x.device, dtype=torch.bfloat16)
    r2 = _as_rows(residual) if residual is not None else None
    native().skinny_gemm(x2, w, out, r2)
    return out.view(*x.shape[:-1], w.shape[0])


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual):
        x2 = _as_rows(x)
        M, N = x2.shape[0], w.shape[0]
        out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
        r2 = _as_rows(residual) if residual is not None else None
        native().gemm(x2, w, out, r2, 0, 0, 1.0, 1.0 if r2 is not None else 0.0, 0)
        ctx.save_for_backward(x2, w)
        ctx.has_res = residual is not None
        ctx.x_shape = x.shape
        return out.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = _as_rows(dy)
        dx = dw = None
        C = native()
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x2)
            C.gemm(dy2, w, dx, None, 0, 1, 1.0, 0.0, 0)
            dx = dx.view(ctx.x_shape)
        if ctx.needs_input_grad[1]:
            dw = torch.empty_like(w)
            C.gemm(dy2, x2, dw, None, 1, 1, 1.0, 0.0, 0)
        dres = dy if ctx.has_res else None
        return dx, dw, dres


def pack_params(params) -> torch.Tensor:
    """Make the 2-D parameters ``params`` (same in-dim) views of ONE contiguous
    buffer, in order, and return the buffer. Parameter objects are kept (only
    ``.data`` is re-pointed), so optimizers and state dicts are unaffected."""
    params = list(params)
    base = params[0]
    if len(params) > 1 and _packed(params):
        return _packed_view(params)
    rows = sum(p.shape[0] for p in params)
    # parameters must stay normal tensors even when first packed under inference_mode (a rollout
    # before any training step): a buffer made there could never be saved for backward
    with torch.inference_mode(False):
        buf = torch.empty((rows, base.shape[1]), device=base.device, dtype=base.dtype)
    r = 0
    with torch.inference_mode(False), torch.no_grad():
        for p in params:
            n = p.shape[0]
            buf[r:r + n].copy_(p.data)
            p.data = buf[r:r + n]
            r += n
    return buf


def _packed(params) -> bool:
    p0 = params[0]
    if not p0.is_contiguous():
        return False
    ptr = p0.data_ptr()
    for p in params:
        if p.data_ptr() != ptr or not p.is_contiguous() or p.dtype != p0.dtype or p.shape[1] != p0.shape[1] \
                or p.untyped_storage().data_ptr() != p0.untyped_storage().data_ptr():
            return False
        ptr += p.numel() * p.element_size()
    return True


def _packed_view(params) -> torch.Tensor:
    p0 = params[0]
    rows = sum(p.shape[0] for p in params)
    return p0.data.as_strided((rows, p0.shape[1]), (p0.shape[1], 1))


class _PackedLinearFn(torch.autograd.Function):
    """y = x @ W^T (+ residual) with W = rows of the packed parameters.

    The weight gradient is written by the GEMM straight into a packed
    gradient buffer whose row slices are the parameters' ``.grad`` tensors:
    the first micro-batch after ``zero_grad`` overwrites (beta = 0), later
    ones accumulate in the GEMM epilogue (beta = 1). No autograd
    accumulation kernels, no split copies."""

    @staticmethod
    def forward(ctx, x, w, residual, *params):
        x2 = _as_rows(x)
        M, N = x2.shape[0], w.shape[0]
        out = torch.empty((M, N), device=x.device, dtype=torch.bfloat16)
        r2 = _as_rows(residual) if residual is not None else None
        native().gemm(x2, w, out, r2, 0, 0, 1.0, 1.0 if r2 is not None else 0.0, 0)
        ctx.save_for_backward(x2, w)
        ctx.params = params
        ctx.has_res = residual is not None
        ctx.x_shape = x.shape
        return out.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = _as_rows(dy)
        C = native()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x2)
            C.gemm(dy2, w, dx, None, 0, 1, 1.0, 0.0, 0)
            dx = dx.view(ctx.x_shape)
        accumulate_weight_grad(dy2, x2, w, ctx.params)
        dres = dy if ctx.has_res else None
        return (dx, None, dres) + (None,) * len(ctx.params)


def accumulate_weight_grad(dy2: torch.Tensor, x2: torch.Tensor, w: torch.Tensor, params) -> None:
    """``params[i].grad += rows of dy2^T x2`` (the weight gradient of ``x2 @ cat(params)^T``).

    The first micro-batch after ``zero_grad`` writes one packed gradient buffer whose row slices
    become the ``.grad`` tensors (beta 0); later micro-batches accumulate in the GEMM epilogue
    (beta 1), so gradient accumulation costs no extra kernel."""
    C = native()
    live = [p for p in params if p.requires_grad]
    if not live:
        return
    if live[0].grad is None:
        buf = torch.empty_like(w)
        C.gemm(dy2, x2, buf, None, 1, 1, 1.0, 0.0, 0)
        r = 0
        for p in params:
            n = p.shape[0]
            if p.requires_grad:
                p.grad = buf[r:r + n]
            r += n
        return
    grads = [p.grad for p in params]
    if all(g is not None for g in grads) and _packed(grads):
        buf = _packed_view(grads)
        C.gemm(dy2, x2, buf, buf, 1, 1, 1.0, 1.0, 0)
        return
    tmp = torch.empty_like(w)  # foreign gradient layout: compute and add
    C.gemm(dy2, x2, tmp, None, 1, 1, 1.0, 0.0, 0)
    r = 0
    for p in params:
        n = p.shape[0]
        if p.requires_grad:
            p.grad = tmp[r:r + n].clone() if p.grad is None else p.grad.add_(tmp[r:r + n])
        r += n


class _SwiGLUMLPFn(torch.autograd.Function):
    """``down(up(x) * silu(gate(x))) + residual`` with the SwiGLU in GEMM epilogues.

    Forward: one GEMM whose tiles pair 128 up rows with the matching 128 gate rows of the packed
    weight writes h = (u, g) and a = silu(g) * u; a second GEMM applies down (+ residual).
    Backward: the down data-gradient GEMM turns da into dh = (da * silu(g), da * u * silu'(g)) in
    its epilogue (da is never stored), then dx = dh W_ug and the three weight gradients."""

    @staticmethod
    def forward(ctx, x, w_ug, w_down, residual, n_ug, *params):
        C = native()
        x2 = _as_rows(x)
        M, F_ = x2.shape[0], w_ug.shape[0] // 2
        h = torch.empty((M, 2 * F_), device=x.device, dtype=torch.bfloat16)
        a = torch.empty((M, F_), device=x.device, dtype=torch.bfloat16)
        C.gemm_swiglu(1, x2, w_ug, h, a, None)
        D = w_down.shape[0]
        out = torch.empty((M, D), device=x.device, dtype=torch.bfloat16)
        r2 = _as_rows(residual) if residual is not None else None
        C.gemm(a, w_down, out, r2, 0, 0, 1.0, 1.0 if r2 is not None else 0.0, 0)
        ctx.save_for_backward(x2, w_ug, w_down, h, a)
        ctx.n_ug, ctx.params, ctx.has_res, ctx.x_shape = n_ug, params, residual is not None, x.shape
        return out.view(*x.shape[:-1], D)

    @staticmethod
    def backward(ctx, dy):
        x2, w_ug, w_down, h, a = ctx.saved_tensors
        C = native()
        dy2 = _as_rows(dy)
        ug, dn = ctx.params[:ctx.n_ug], ctx.params[ctx.n_ug:]
        accumulate_weight_grad(dy2, a, w_down, dn)
        dh = torch.empty_like(h)
        C.gemm_swiglu(2, dy2, w_down, None, dh, h)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x2)
            C.gemm(dh, w_ug, dx, None, 0, 1, 1.0, 0.0, 0)
            dx = dx.view(ctx.x_shape)
        accumulate_weight_grad(dh, x2, w_ug, ug)
        dres = dy if ctx.has_res else None
        return (dx, None, None, dres, None) + (None,) * len(ctx.params)


def swiglu_mlp(x: torch.Tensor, up: torch.Tensor, gate: torch.Tensor, down: torch.Tensor,
               residual: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Fused SwiGLU MLP on the kernel path, or None when it does not apply (then compose
    :func:`packed_linear`, :func:`astrai_b200.ops.activation.swiglu` and :func:`linear`)."""
    params = (up, gate, down)
    no_grad = not torch.is_grad_enabled() or not (x.requires_grad or any(p.requires_grad for p in params))
    if not PACKING or not (INFER_SWIGLU if no_grad else FUSED_SWIGLU):
        return None
    if not (x.is_cuda and x.dtype == torch.bfloat16 and all(
            p.is_cuda and p.dtype == torch.bfloat16 and type(p.data) is torch.Tensor for p in params)):
        return None
    F_, d = up.shape
    if F_ % 128 or (d * 2) % 16 or down.shape != (d, F_) or x.shape[-1] != d:
        return None
    if no_grad and x.reshape(-1, d).shape[0] <= SKINNY_MAX_ROWS:
        return None  # decode rows: the skinny kernels stream each weight once
    w_ug = pack_params([up, gate])
    if no_grad:
        C = native()
        x2 = _as_rows(x)
        a = torch.empty((x2.shape[0], F_), device=x.device, dtype=torch.bfloat16)
        C.gemm_swiglu(1, x2, w_ug.detach(), None, a, None)
        out = torch.empty((x2.shape[0], d), device=x.device, dtype=torch.bfloat16)
        r2 = _as_rows(residual) if residual is not None else None
        C.gemm(a, down.detach(), out, r2, 0, 0, 1.0, 1.0 if r2 is not None else 0.0, 0)
        return out.view(*x.shape[:-1], d)
    return _SwiGLUMLPFn.apply(x, w_ug.detach(), down.detach(), residual, 2, up, gate, down)


class _PackedLinearRopeFn(torch.autograd.Function):
    """``rope(x @ cat(params)^T)`` on the first ``rope_cols`` columns, the rotation applied in the GEMM
    epilogue; backward rotates the incoming gradient back (in place) before the usual products."""

    @staticmethod
    def forward(ctx, x, w, table, positions, seq_len, rope_cols, head_dim, *params):
        x2 = _as_rows(x)
        out = torch.empty((x2.shape[0], w.shape[0]), device=x.device, dtype=torch.bfloat16)
        native().gemm_rope(x2, w, out, table, positions, seq_len, rope_cols, head_dim)
        ctx.save_for_backward(x2, w, table, positions)
        ctx.params, ctx.x_shape, ctx.rope = params, x.shape, (seq_len, rope_cols, head_dim)
        return out.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        from astrai_b200.ops.rope import rope_inplace

        x2, w, table, positions = ctx.saved_tensors
        seq_len, rope_cols, head_dim = ctx.rope
        # the gradient arriving here is the attention kernel's fresh dqkv buffer (the projection's
        # only consumer), so it is rotated back in place
        dy2 = _as_rows(dy)
        rope_inplace(dy2, 0, rope_cols // head_dim, head_dim, table, positions, seq_len, inverse=True)
        C = native()
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty_like(x2)
            C.gemm(dy2, w, dx, None, 0, 1, 1.0, 0.0, 0)
            dx = dx.view(ctx.x_shape)
        accumulate_weight_grad(dy2, x2, w, ctx.params)
        return (dx, None, None, None, None, None, None) + (None,) * len(ctx.params)


def packed_linear_rope(x: torch.Tensor, params, table: torch.Tensor, positions: Optional[torch.Tensor],
                       seq_len: int, rope_cols: int, head_dim: int) -> Optional[torch.Tensor]:
    """Packed projection with interleaved RoPE on its first ``rope_cols`` output columns (the q and k heads
    of a fused QKV projection), or None when the kernel path does not apply."""
    params = list(params)
    if not FUSED_ROPE or not PACKING:
        return None
    if not (x.is_cuda and x.dtype == torch.bfloat16 and all(
            p.is_cuda and p.dtype == torch.bfloat16 and type(p.data) is torch.Tensor for p in params)):
        return None
    if (x.shape[-1] * 2) % 16 or head_dim % 32 or rope_cols % head_dim:
        return None
    w = pack_params(params) if len(params) > 1 else params[0]
    if not torch.is_grad_enabled() or not (x.requires_grad or any(p.requires_grad for p in params)):
        x2 = _as_rows(x)
        if x2.shape[0] <= SKINNY_MAX_ROWS:
            return None  # decode rows: the skinny GEMM and the cache's own RoPE
        out = torch.empty((x2.shape[0], w.shape[0]), device=x.device, dtype=torch.bfloat16)
        native().gemm_rope(x2, w.detach(), out, table, positions, seq_len, rope_cols, head_dim)
        return out.view(*x.shape[:-1], w.shape[0])
    return _PackedLinearRopeFn.apply(x, w.detach(), table, positions, seq_len, rope_cols, head_dim, *params)


def packed_linear(x: torch.Tensor, params, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``x @ cat(params)^T (+ residual)`` for bias-free 2-D bf16 parameters.

    On CUDA the parameters are packed once into one contiguous weight (views),
    so no concatenation happens per call, and weight gradients accumulate in
    the GEMM epilogue. Parameters held as DTensors (FSDP) or on the CPU take
    the autograd path of :func:`linear`."""
    params = list(params)
    cuda_ok = x.is_cuda and x.dtype == torch.bfloat16 and all(
        p.is_cuda and p.dtype == torch.bfloat16 and type(p.data) is torch.Tensor for p in params)
    if not cuda_ok or (x.shape[-1] * 2) % 16 or (len(params) > 1 and not PACKING):
        w = params[0] if len(params) == 1 else torch.cat(list(params), 0)
        return linear(x, w, residual=residual)
    w = pack_params(params) if len(params) > 1 else params[0]
    y = _skinny(x, w.detach(), residual)
    if y is not None:
        return y
    return _PackedLinearFn.apply(x, w.detach(), residual, *params)


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None,
           bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w.T (+ bias) (+ residual)."""
    if (not x.is_cuda) or bias is not None or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 \
            or (x.shape[-1] * 2) % 16 or (w.shape[0] * 2) % 16:
        # CPU oracle path (and odd dtypes / shapes that TMA cannot address)
        if x.is_cuda and x.dtype == torch.bfloat16 and bias is None:
            raise ValueError(f"linear: dims {tuple(x.shape)} x {tuple(w.shape)} need 16-byte aligned rows")
        y = F.linear(x, w, bias)
        return y + residual if residual is not None else y
    y = _skinny(x, w, residual)
    if y is not None:
        return y
    return _LinearFn.apply(x, w, residual)
