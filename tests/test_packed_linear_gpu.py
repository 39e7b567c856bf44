"""Packed projection weights (views of one buffer) and GEMM-epilogue gradient
accumulation across micro-batches, against plain fp32 autograd."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_packed_linear_accumulates_like_autograd():
    from astrai_b200.ops.gemm import packed_linear

    torch.manual_seed(0)
    ws = [torch.nn.Parameter((torch.randn(n, 256, device="cuda") * 0.05).to(torch.bfloat16)) for n in (256, 128, 128)]
    ref = [torch.nn.Parameter(w.detach().float().clone()) for w in ws]
    xs = [torch.randn(3, 64, 256, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    gs = [torch.randn(3, 64, 512, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    for x, g in zip(xs, gs):
        packed_linear(x, ws).backward(g)
        (x.float() @ torch.cat(ref).t()).backward(g.float())
    ptr = ws[0].data_ptr()
    for w in ws:  # parameters are now contiguous views of one buffer
        assert w.data_ptr() == ptr
        ptr += w.numel() * 2
    for w, r in zip(ws, ref):
        err = ((w.grad.float() - r.grad).norm() / r.grad.norm()).item()
        assert err < 1e-2
