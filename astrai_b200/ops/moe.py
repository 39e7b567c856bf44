"""MoE autograd ops: fused router and the (expert-parallel) routed-expert block.

``moe_route(logits, k)`` -> (weights [T, k] fp32, probs [T, E] fp32, idx, counts, pos)
runs the router kernel (fp32 softmax, top-k, renormalisation, per-expert slot
tickets); its backward is closed-form on the small [T, E] tensors.

``moe_experts(...)`` runs dispatch -> grouped expert GEMMs (up|gate, SwiGLU,
down; each expert's rows padded to whole 128-row tiles, tiles past the live
rows skipped, so work follows the actual expert loads) -> return -> weighted combine with an additive input
(residual + shared experts) in the forward, and the mirror image in the
backward: combine-backward (gate-weight gradients + scaled output gradients
pushed to the expert ranks) -> grouped dgrad / per-expert-K wgrad GEMMs ->
return of the input gradients -> sum over slots. Expert weights are the stacked views made by
:func:`stack_expert_params`; their gradients are written (or accumulated,
beta = 1) by the weight-gradient GEMMs directly into stacked gradient buffers
whose slices are the parameters' ``.grad``.
"""

from __future__ import annotations

from typing import List, Sequence

import torch

from astrai_b200.ops._ext import native
from astrai_b200.ops.gemm import _packed, _packed_view, pack_params
from astrai_b200.parallel.ep import PH_DISPATCH, PH_RETURN, PH_RETURN_BWD, PH_SCATTER_BWD, EPArena, EPLayout


class _RouterFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, k):
        C = native()
        T, E = logits.shape
        dev = logits.device
        probs = torch.empty((T, E), device=dev, dtype=torch.float32)
        idx = torch.empty((T, k), device=dev, dtype=torch.int32)
        w = torch.empty((T, k), device=dev, dtype=torch.float32)
        counts = torch.zeros(E, device=dev, dtype=torch.int32)
        pos = torch.empty(T * k, device=dev, dtype=torch.int32)
        C.moe_router(logits if logits.stride(-1) == 1 else logits.contiguous(), k, probs, idx, w, counts, pos)
        ctx.save_for_backward(probs, idx, w)
        ctx.dtype = logits.dtype
        ctx.mark_non_differentiable(idx, counts, pos)
        return w, probs, idx, counts, pos

    @staticmethod
    def backward(ctx, dw, dprobs, *_):
        probs, idx, w = ctx.saved_tensors
        dp = dprobs.float().clone() if dprobs is not None else torch.zeros_like(probs)
        if dw is not None:
            # w_j = p_j / S (S = sum of the selected probabilities)
            sel = probs.gather(1, idx.long())
            S = sel.sum(-1, keepdim=True)
            dwf = dw.float()
            g = (dwf - (dwf * w).sum(-1, keepdim=True)) / S
            dp.scatter_add_(1, idx.long(), g)
        dlogits = probs * (dp - (probs * dp).sum(-1, keepdim=True))
        return dlogits.to(ctx.dtype), None


def moe_route(logits: torch.Tensor, k: int):
    return _RouterFn.apply(logits, k)


def stack_expert_params(experts) -> tuple:
    """Views of the local experts' weights as stacked tensors:
    ``W_gu [E, 2F, d]`` (rows: up then gate of each expert) and ``W_dn [E, d, F]``."""
    up_gate: List[torch.nn.Parameter] = []
    down: List[torch.nn.Parameter] = []
    for m in experts:
        up_gate += [m.up.weight, m.gate.weight]
        down.append(m.down.weight)
    E = len(down)
    F, d = up_gate[0].shape
    w_gu = pack_params(up_gate).view(E, 2 * F, d)
    w_dn = pack_params(down).view(E, d, F)
    return w_gu, w_dn, up_gate, down


def _stacked_grad(params: Sequence[torch.nn.Parameter], shape, compute) -> None:
    """Write / accumulate a stacked weight gradient computed by ``compute(out, beta)``."""
    grads = [p.grad for p in params]
    if all(g is None for g in grads):
        buf = torch.empty(shape, device=params[0].device, dtype=params[0].dtype)
        compute(buf, 0.0)
        flat = buf.view(-1, params[0].shape[1])
        r = 0
        for p in params:
            n = p.shape[0]
            p.grad = flat[r:r + n]
            r += n
    elif all(g is not None for g in grads) and _packed(grads):
        compute(_packed_view(grads).view(shape), 1.0)
    else:
        tmp = torch.empty(shape, device=params[0].device, dtype=params[0].dtype)
        compute(tmp, 0.0)
        flat = tmp.view(-1, params[0].shape[1])
        r = 0
        for p in params:
            n = p.shape[0]
            p.grad = flat[r:r + n].clone() if p.grad is None else p.grad.add_(flat[r:r + n])
            r += n


class _ExpertsFn(torch.autograd.Function):
    """Routed experts over the arena's capacity-sized blocks (``R = arena.rows_cap`` rows); the live
    rows, their experts and the tiles to skip come from the device-side layout, so no value is read
    back to the host."""

    @staticmethod
    def forward(ctx, x, add, w, idx, pos, w_gu, w_dn, arena: EPArena, layout: EPLayout, n_ug: int, *params):
        C = native()
        T, d = x.shape
        k = idx.shape[1]
        El, R = layout.e_local, layout.rows
        F = w_dn.shape[2]
        dev = x.device
        slot_row = torch.empty(T * k, device=dev, dtype=torch.int32)
        dispatch = C.ep_dispatch_fp8 if arena.fp8 else C.ep_dispatch
        dispatch(*arena.args(), x, idx.view(-1), pos, layout.base_row, El, slot_row)
        C.ep_wait(*arena.args(), PH_DISPATCH)
        if arena.fp8:
            C.ep_dequant(*arena.args(), R)
        h = torch.empty((R, 2 * F), device=dev, dtype=torch.bfloat16)
        a = torch.empty((R, F), device=dev, dtype=torch.bfloat16)
        y = torch.empty((R, d), device=dev, dtype=torch.bfloat16)
        xin = arena.block("xin", R)
        C.gemm_grouped(0, xin, w_gu, h, group_tile=layout.group_tile)
        C.swiglu_fwd(h, a, layout.total)
        C.gemm_grouped(0, a, w_dn, y, group_tile=layout.group_tile)
        C.ep_return(*arena.args(), y, layout.group_tile, layout.starts, layout.n_rows, 0)
        C.ep_wait(*arena.args(), PH_RETURN)
        out = torch.empty((T, d), device=dev, dtype=torch.bfloat16)
        C.ep_combine(arena.block("ret", T * k), w, add, out, k)
        ctx.save_for_backward(w, idx, slot_row, w_gu, w_dn, h, a)
        ctx.arena, ctx.layout, ctx.n_ug, ctx.params = arena, layout, n_ug, params
        ctx.dims = (T, d, k, F)
        return out

    @staticmethod
    def backward(ctx, dout):
        C = native()
        w, idx, slot_row, w_gu, w_dn, h, a = ctx.saved_tensors
        arena, layout = ctx.arena, ctx.layout
        T, d, k, F = ctx.dims
        El, R = layout.e_local, layout.rows
        dev = dout.device
        dout = dout.contiguous()
        dw = torch.empty((T, k), device=dev, dtype=torch.float32)
        C.ep_zero_pad(*arena.args(), 1, R, layout.group_tile, layout.starts, layout.n_rows)
        C.ep_combine_bwd(*arena.args(), dout, arena.block("ret", T * k), w, idx.view(-1), slot_row, El, dw)
        C.ep_wait(*arena.args(), PH_SCATTER_BWD)
        ug, dn = ctx.params[:ctx.n_ug], ctx.params[ctx.n_ug:]
        dy = arena.block("dyin", R)
        xin = arena.block("xin", R)
        da = torch.empty((R, F), device=dev, dtype=torch.bfloat16)
        C.gemm_grouped(0, dy, w_dn, da, group_tile=layout.group_tile, b_mn=1)
        # weight gradients over each expert's padded row range (an expert with no rows: k_count 0
        # writes beta * C, i.e. zeros on the first micro-batch and no change after)
        if any(p.requires_grad for p in dn):
            _stacked_grad(dn, (El, d, F), lambda out, beta: C.gemm_grouped(
                1, dy, a, out, out if beta else None, k_start=layout.starts, k_count=layout.k_count, beta=beta))
        dh = torch.empty((R, 2 * F), device=dev, dtype=torch.bfloat16)
        C.swiglu_bwd(da, h, dh, layout.total)
        if any(p.requires_grad for p in ug):
            _stacked_grad(ug, (El, 2 * F, d), lambda out, beta: C.gemm_grouped(
                1, dh, xin, out, out if beta else None, k_start=layout.starts, k_count=layout.k_count, beta=beta))
        dxin = torch.empty((R, d), device=dev, dtype=torch.bfloat16)
        C.gemm_grouped(0, dh, w_gu, dxin, group_tile=layout.group_tile, b_mn=1)
        C.ep_return(*arena.args(), dxin, layout.group_tile, layout.starts, layout.n_rows, 1)
        C.ep_wait(*arena.args(), PH_RETURN_BWD)
        dx = torch.empty((T, d), device=dev, dtype=torch.bfloat16)
        C.ep_combine(arena.block("ret2", T * k), None, None, dx, k)
        return (dx, dout, dw, None, None, None, None, None, None, None) + (None,) * len(ctx.params)


def moe_experts(x, add, w, idx, pos, experts_stack, arena: EPArena, layout: EPLayout):
    """Routed-expert block: ``add + sum_j w[:, j] * expert_{idx[:, j]}(x)``."""
    w_gu, w_dn, ug, dn = experts_stack
    return _ExpertsFn.apply(x, add, w, idx, pos, w_gu.detach(), w_dn.detach(), arena, layout, len(ug), *ug, *dn)
