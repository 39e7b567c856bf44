"""Runs each hot kernel of the framework once on a case larger than L2, for profiler captures.

``python -m astrai_b200.utils.kernel_cases [ce rope swiglu gemm_swiglu gemm_swiglu_train gemm_rope embedding router sample decode adamw muon ep]``
(no argument: all of them). One launch per kernel (two for the forward/backward pairs), shapes of
the 1.1B dense step (8192 tokens, d 2048, FFN 5632, vocab 32000), the MoE layer (64 experts top-6,
one-rank expert-parallel group) and batch-32 decode over a 4096-token paged cache, so an ``ncu``
capture of one kernel each (``-k regex:... -c N``) reads DRAM figures that mean something and ends
in seconds. Exits non-zero if a kernel raised the device error word.
"""

import math
import sys

import torch


def run(which):
    from astrai_b200.ops._ext import native

    C = native()
    dev = "cuda"
    torch.manual_seed(0)

    def want(n):
        return "all" in which or n in which

    if want("ce"):
        from astrai_b200.ops.loss import cross_entropy
        logits = (torch.randn(8192, 32000, device=dev) * 2).to(torch.bfloat16).requires_grad_()
        tgt = torch.randint(0, 32000, (8192,), device=dev)
        cross_entropy(logits, tgt, label_smoothing=0.1).backward()
        del logits
    if want("rope"):
        from astrai_b200.ops.rope import rope_inplace, rope_table
        tab = rope_table(128, 2048, 1e6, device=dev)
        qkv = torch.randn(8192, 24 * 128, device=dev).to(torch.bfloat16)
        rope_inplace(qkv, 0, 20, 128, tab, None, 2048)
    if want("swiglu"):
        from astrai_b200.ops.activation import swiglu
        h = torch.randn(8192, 11264, device=dev).to(torch.bfloat16).requires_grad_()
        a = swiglu(h)
        a.backward(torch.randn_like(a))
        del h, a
    if want("gemm_swiglu"):
        # the up/gate projection of a 2048-token prefill at d 1536, FFN 6912: the plain GEMM writing
        # h = (u, g), then the SwiGLU-epilogue GEMM writing only a = silu(g) * u
        x = torch.randn(2048, 1536, device=dev).to(torch.bfloat16)
        w = (torch.randn(2 * 6912, 1536, device=dev) * 0.02).to(torch.bfloat16)
        h = torch.empty(2048, 2 * 6912, device=dev, dtype=torch.bfloat16)
        a = torch.empty(2048, 6912, device=dev, dtype=torch.bfloat16)
        C.gemm(x, w, h, None, 0, 0, 1.0, 0.0, 0)
        C.gemm_swiglu(1, x, w, None, a, None)
        del x, w, h, a
    if want("gemm_swiglu_train"):
        # the 1.1B step's up/gate projection (8192 tokens, d 2048, FFN 5632): the plain GEMM writing
        # h, then the SwiGLU-epilogue GEMM writing h and a (what training would store)
        x = torch.randn(8192, 2048, device=dev).to(torch.bfloat16)
        w = (torch.randn(2 * 5632, 2048, device=dev) * 0.02).to(torch.bfloat16)
        h = torch.empty(8192, 2 * 5632, device=dev, dtype=torch.bfloat16)
        a = torch.empty(8192, 5632, device=dev, dtype=torch.bfloat16)
        C.gemm(x, w, h, None, 0, 0, 1.0, 0.0, 0)
        C.gemm_swiglu(1, x, w, h, a, None)
        del x, w, h, a
    if want("gemm_rope"):
        # the 1.1B step's QKV projection (8192 tokens, d 2048 -> 16 + 4 + 4 heads of 128): the plain
        # GEMM, then the GEMM with RoPE on the q and k columns in its epilogue
        from astrai_b200.ops.rope import rope_table
        x = torch.randn(8192, 2048, device=dev).to(torch.bfloat16)
        w = (torch.randn(3072, 2048, device=dev) * 0.02).to(torch.bfloat16)
        y = torch.empty(8192, 3072, device=dev, dtype=torch.bfloat16)
        tab = rope_table(128, 2048, 1e6, device=dev)
        C.gemm(x, w, y, None, 0, 0, 1.0, 0.0, 0)
        C.gemm_rope(x, w, y, tab, None, 2048, 20 * 128, 128)
        del x, w, y
    if want("embedding"):
        from astrai_b200.ops.embedding import embedding
        w = (torch.randn(32000, 2048, device=dev) * 0.02).to(torch.bfloat16).requires_grad_()
        ids = torch.randint(0, 32000, (4, 2048), device=dev)
        e = embedding(ids, w)
        e.backward(torch.randn_like(e))
    if want("router"):
        from astrai_b200.ops.moe import moe_route
        lg = torch.randn(16384, 64, device=dev).requires_grad_()
        w, probs, idx, counts, pos = moe_route(lg, 6)
    if want("sample"):
        from astrai_b200.inference.sample import sample
        sample(torch.randn(4, 32000, device=dev) * 3, temperature=0.8, top_k=50, top_p=0.95)
    if want("decode"):
        B, Hq, Hkv, page, L = 32, 32, 4, 128, 4096
        n_pages = B * L // page
        kc = torch.randn(n_pages, Hkv, page, 128, device=dev).to(torch.bfloat16)
        vc = torch.randn_like(kc)
        table = torch.arange(n_pages, device=dev, dtype=torch.int32).view(B, L // page)
        lens = torch.full((B,), L, device=dev, dtype=torch.int32)
        q = torch.randn(B, Hq * 128, device=dev).to(torch.bfloat16)
        out = torch.empty_like(q)
        splits = int(C.decode_splits(B, Hkv, L, 0))
        ws = torch.empty(B * Hq * splits * 130, device=dev)
        C.paged_decode(q, kc, vc, table, lens, out, Hq, 1 / math.sqrt(128), splits, ws)
    if want("adamw"):
        from astrai_b200.optim import FusedAdamW
        ps = [torch.nn.Parameter((torch.randn(4096, 4096, device=dev) * 0.02).to(torch.bfloat16)) for _ in range(4)]
        for p in ps: p.grad = torch.randn_like(p) * 1e-3
        FusedAdamW(ps, lr=1e-4, weight_decay=0.1).step()
    if want("muon"):
        from astrai_b200.optim.fused import Muon
        ps = [torch.nn.Parameter((torch.randn(2048, 5632, device=dev) * 0.02).to(torch.bfloat16)) for _ in range(8)]
        for p in ps: p.grad = torch.randn_like(p) * 1e-3
        Muon(ps, lr=0.02, adjust_lr_fn="match_rms_adamw").step()
    if want("ep"):
        from astrai_b200.parallel.ep import PH_DISPATCH, PH_RETURN, EPArena, EPGroup
        T, d, k, E = 8192, 2048, 6, 64
        idx = torch.randint(0, E, (T, k), device=dev, dtype=torch.int32)
        counts = torch.bincount(idx.view(-1).long(), minlength=E)
        order = torch.argsort(idx.view(-1).long(), stable=True)
        pos = torch.empty(T * k, device=dev, dtype=torch.int64)
        starts = torch.cumsum(counts, 0) - counts
        pos[order] = torch.arange(T * k, device=dev) - starts.repeat_interleave(counts)
        pos = pos.to(torch.int32)
        x = torch.randn(T, d, device=dev).to(torch.bfloat16)
        arena = EPArena(EPGroup.local(), d, T, k, E, 2.0, torch.device(dev))
        layout = arena.compute_layout(counts.to(torch.int32))
        slot_row = torch.empty(T * k, device=dev, dtype=torch.int32)
        C.ep_dispatch(*arena.args(), x, idx.view(-1), pos, layout.base_row, E, slot_row)
        C.ep_wait(*arena.args(), PH_DISPATCH)
        y = arena.block("xin", layout.rows).clone()
        C.ep_return(*arena.args(), y, layout.group_tile, layout.starts, layout.n_rows, 0)
        C.ep_wait(*arena.args(), PH_RETURN)
        w = torch.rand(T, k, device=dev)
        out = torch.empty(T, d, device=dev, dtype=torch.bfloat16)
        C.ep_combine(arena.block("ret", T * k), w, None, out, k)
        torch.cuda.synchronize()
        arena.close()
    torch.cuda.synchronize()
    err = C.read_error()
    if err:
        raise SystemExit(f"device error word {err:#x}")
    print("ok", which)


def main(argv=None):
    which = list(argv if argv is not None else sys.argv[1:]) or ["all"]
    run(which)


if __name__ == "__main__":
    main()
