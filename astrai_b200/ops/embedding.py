"""Token embedding gather / scatter-add (parity: astrai/model/components/embedding.py:21-26)."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from astrai_b200.ops._ext import native


class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        ids_c = ids.contiguous().long()
        out = torch.empty((*ids.shape, w.shape[1]), device=w.device, dtype=w.dtype)
        native().embedding_fwd(ids_c.view(-1), w, out.view(-1, w.shape[1]))
        ctx.save_for_backward(ids_c)
        ctx.wshape = w.shape
        return out

    @staticmethod
    def backward(ctx, g):
        (ids_c,) = ctx.saved_tensors
        C = native()
        acc = torch.zeros(ctx.wshape, device=g.device, dtype=torch.float32)
        C.embedding_bwd(ids_c.view(-1), g.reshape(-1, ctx.wshape[1]).contiguous(), acc)
        dw = torch.empty(ctx.wshape, device=g.device, dtype=torch.bfloat16)
        C.f32_to_bf16(acc, dw, False)
        return None, dw


def embedding(ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    if weight.is_cuda and weight.dtype == torch.bfloat16 and weight.shape[1] % 8 == 0:
        return _EmbeddingFn.apply(ids, weight)
    return F.embedding(ids, weight)
