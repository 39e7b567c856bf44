"""Device-timed micro-benchmarks of the framework's kernels.

    python -m astrai_b200.utils.kernel_bench [gemm [case]|gemm_shapes|swiglu_gemm|rope_gemm|elementwise|ns|attn|norm|skinny|sample|decode|prefill|all]
    torchrun --nproc-per-node N -m astrai_b200.utils.kernel_bench allreduce|ep|tpgather|tprow

Each case is timed with CUDA events on the launching stream after warm-up,
with a synchronize on both sides; inputs larger than L2 are used where the
op is bandwidth-bound. Prints one JSON line per case with the achieved rate
and its fraction of the measured peaks (MEASURED_PEAKS.json when present,
else the pool's fallback figures).
"""

from __future__ import annotations

import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def time_fn(fn, warmup=5, iters=20):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(only=None):
    """The GEMMs of the 1.1B training step (``only``: one case by name, e.g. for a profiler capture)."""
    from astrai_b200.ops._ext import native

    hbm, tf, src = peaks()
    C = native()
    cases = [
        # name, M, N, K, a_mn, b_mn  (1.1B dense config, 4 x 2048 tokens)
        ("qkv_fwd", 8192, 3072, 2048, 0, 0),
        ("o_fwd", 8192, 2048, 2048, 0, 0),
        ("upgate_fwd", 8192, 11264, 2048, 0, 0),
        ("down_fwd", 8192, 2048, 5632, 0, 0),
        ("lm_head_fwd", 8192, 32000, 2048, 0, 0),
        ("down_dgrad", 8192, 5632, 2048, 0, 1),
        ("upgate_wgrad", 11264, 2048, 8192, 1, 1),
        ("o_wgrad", 2048, 2048, 8192, 1, 1),
        ("qkv_wgrad", 3072, 2048, 8192, 1, 1),
        ("square_8192", 8192, 8192, 8192, 0, 0),
    ]
    for name, M, N, K, amn, bmn in cases:
        if only is not None and name != only:
            continue
        a = torch.randn((K, M) if amn else (M, K), device="cuda", dtype=torch.bfloat16)
        b = torch.randn((K, N) if bmn else (N, K), device="cuda", dtype=torch.bfloat16)
        d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: C.gemm(a, b, d, None, amn, bmn, 1.0, 0.0, 0))  # automatic plan
        A = a.t() if amn else a
        B = b if bmn else b.t()
        ms_ref = time_fn(lambda: torch.matmul(A, B))
        # the single-CTA kernel (force_bn 2: its automatic tile shape, Stream-K where it applies)
        # and its largest deviation from the automatic plan's output
        d2 = torch.empty_like(d)
        ms_1cta = time_fn(lambda: C.gemm(a, b, d2, None, amn, bmn, 1.0, 0.0, 2))
        dev = float((d2.float() - d.float()).abs().max() / d.float().abs().max().clamp_min(1e-30))
        fl = 2.0 * M * N * K
        # one extra launch of the single-CTA kernel with its wait-cycle counters on: where it stalls
        cnt = torch.zeros(4, device="cuda", dtype=torch.int64)
        C.gemm_profile_set(cnt)
        C.gemm(a, b, d, None, amn, bmn, 1.0, 0.0, 2)
        torch.cuda.synchronize()
        C.gemm_profile_set(None)
        w = [int(v) for v in cnt.tolist()]
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        cyc = ms_1cta * 1e-3 * 1.9e9  # cycles of one CTA at ~1.9 GHz
        bm, bn, streamk, tiles, _, pair, pair_sk = C.gemm_plan(M, N, K, 1)
        ms_pair_sk = time_fn(lambda: C.gemm(a, b, d2, None, amn, bmn, 1.0, 0.0, 1026))  # pair + Stream-K
        print(json.dumps({"kernel": "gemm", "case": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                          "pair": pair, "pair_streamk_applies": pair_sk, "pair_streamk_ms": round(ms_pair_sk, 4),
                          "single_cta_tile": f"{bm}x{bn}", "single_cta_tiles": tiles,
                          "single_cta_streamk": streamk,
                          "tflops": round(fl / ms / 1e9, 1), "frac_of_peak": round(fl / ms / 1e9 / tf, 3),
                          "peak_src": src, "cublas_ms": round(ms_ref, 4),
                          "cublas_tflops": round(fl / ms_ref / 1e9, 1),
                          "single_cta_ms": round(ms_1cta, 4), "single_cta_tflops": round(fl / ms_1cta / 1e9, 1),
                          "single_cta_rel_dev": round(dev, 5),
                          "single_cta_wait_frac": {k: round(v / sms / cyc, 3) for k, v in
                                                zip(("producer_empty", "mma_full", "mma_acc_empty", "epi_acc_full"),
                                                    w)}}))


def _dist_init():
    from datetime import timedelta

    import torch.distributed as dist

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist.get_rank(), dist.get_world_size()


def bench_allreduce():
    """Fused NVLink gradient all-reduce vs NCCL (AVG) on 1 GiB of bf16
    gradients in 26 tensors; device time, max over ranks."""
    from datetime import timedelta

    import torch.distributed as dist

    from astrai_b200.parallel.symm import FusedAllReduce

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    W = dist.get_world_size()
    sizes = [2048 * 2048 * 2] * 16 + [32000 * 2048] * 2 + [2048 * 5632 * 3] * 8
    n = sum(sizes)
    grads = [torch.randn(k, device="cuda").to(torch.bfloat16) for k in sizes[:26]]
    n = sum(g.numel() for g in grads)
    def t_max(fn, iters=10):
        ms = time_fn(fn, warmup=3, iters=iters)
        v = torch.tensor([ms], device="cuda")
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v)

    sweep = {}
    for ctas in (32, 74, 148):
        for rnd in (16 << 20, 64 << 20):
            ar = FusedAllReduce(round_elems=rnd, ctas=ctas)
            sweep[f"ctas{ctas}_round{rnd >> 20}M"] = round(t_max(lambda: ar.all_reduce_mean(grads)), 3)
            ar.close()
    best = min(sweep, key=sweep.get)
    fused = sweep[best]

    def nccl():
        for g in grads:
            dist.all_reduce(g, op=dist.ReduceOp.AVG)
    ref = t_max(nccl)
    if dist.get_rank() == 0:
        bytes_ = n * 2
        bus = lambda ms: bytes_ * 2 * (W - 1) / W / (ms / 1e3) / 1e9  # noqa: E731
        print(json.dumps({"kernel": "fused_allreduce", "world": W, "bytes": bytes_, "fused_ms": round(fused, 3),
                          "fused_busbw_gbs": round(bus(fused), 1), "nccl_ms": round(ref, 3),
                          "nccl_busbw_gbs": round(bus(ref), 1), "link_ref_gbs": 770.0, "best": best,
                          "sweep_ms": sweep}))
    dist.destroy_process_group()


def bench_ep(tokens: int = 8192, d: int = 2048, n_experts: int = 64, k: int = 6):
    """Expert-parallel dispatch and combine of one MoE layer's forward (the BASELINE MoE shape:
    seq 4096 x batch 2 tokens per rank, d 2048, 64 experts top-6), our P2P kernels vs an NCCL
    all_to_all_single pipeline moving the same rows; device time, max over ranks.

    dispatch = ep_dispatch + ep_wait (token rows stored into the owning ranks' expert blocks);
    combine = ep_return + ep_wait + ep_combine (expert outputs stored back into the source ranks'
    slot blocks, then the gate-weighted sum). NCCL arm: gather rows by destination rank,
    all_to_all_single, and back with all_to_all_single + a gate-weighted index_add."""
    from datetime import timedelta

    import torch.distributed as dist

    from astrai_b200.ops._ext import native
    from astrai_b200.ops.moe import moe_route
    from astrai_b200.parallel.ep import PH_DISPATCH, PH_RETURN, EPArena, EPGroup

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    C = native()
    ep = EPGroup()
    W, rank = ep.world, ep.rank
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    x = torch.randn(tokens, d, device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn(tokens, n_experts, device=dev, generator=g).to(torch.bfloat16)
    w, _, idx, counts, pos = moe_route(logits, k)
    arena = EPArena(ep, d, tokens, k, n_experts, 2.0, dev)
    arena8 = EPArena(ep, d, tokens, k, n_experts, 2.0, dev, fp8=True)
    layout = arena.compute_layout(counts)  # device-side counts exchange + layout
    layout8 = arena8.compute_layout(counts)
    El, R = layout.e_local, layout.rows
    slot_row = torch.empty(tokens * k, device=dev, dtype=torch.int32)
    y = torch.randn(R, d, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(tokens, d, device=dev, dtype=torch.bfloat16)

    def dispatch():
        C.ep_dispatch(*arena.args(), x, idx.view(-1), pos, layout.base_row, El, slot_row)
        C.ep_wait(*arena.args(), PH_DISPATCH)

    def dispatch_fp8():  # e4m3 rows + 1x128 scales over NVLink, dequantised by the owner
        C.ep_dispatch_fp8(*arena8.args(), x, idx.view(-1), pos, layout8.base_row, El, slot_row)
        C.ep_wait(*arena8.args(), PH_DISPATCH)
        C.ep_dequant(*arena8.args(), R)

    def layout_only():
        arena.compute_layout(counts)

    def combine():
        C.ep_return(*arena.args(), y, layout.group_tile, layout.starts, layout.n_rows, 0)
        C.ep_wait(*arena.args(), PH_RETURN)
        C.ep_combine(arena.block("ret", tokens * k), w, None, out, k)

    # NCCL arm: rows ordered by destination rank (experts are contiguous per rank)
    dest = (idx.view(-1) // El).to(torch.int64)
    order = torch.argsort(dest, stable=True)
    send_counts = torch.bincount(dest, minlength=W)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    tok_of = order // k
    wts = w.reshape(-1)[order].unsqueeze(-1)
    recv = torch.empty(sum(rc), d, device=dev, dtype=torch.bfloat16)
    back = torch.empty(tokens * k, d, device=dev, dtype=torch.bfloat16)

    def nccl_dispatch():
        dist.all_to_all_single(recv, x.index_select(0, tok_of), rc, sc)

    def nccl_combine():
        dist.all_to_all_single(back, recv, sc, rc)
        torch.zeros(tokens, d, device=dev, dtype=torch.float32).index_add_(0, tok_of, back.float() * wts)

    def t_max(fn, iters=20):
        ms = time_fn(fn, warmup=5, iters=iters)
        v = torch.tensor([ms], device=dev)
        dist.all_reduce(v, op=dist.ReduceOp.MAX)
        return float(v) * 1e3  # us

    res = {"layout_us": t_max(layout_only), "dispatch_us": t_max(dispatch), "dispatch_fp8_us": t_max(dispatch_fp8),
           "combine_us": t_max(combine),
           "dispatch_combine_us": t_max(lambda: (dispatch(), combine())),
           "nccl_dispatch_us": t_max(nccl_dispatch), "nccl_combine_us": t_max(nccl_combine),
           "nccl_dispatch_combine_us": t_max(lambda: (nccl_dispatch(), nccl_combine()))}
    from astrai_b200.ops._ext import check_error

    err = check_error()
    # rows that cross NVLink from this rank (slots whose expert lives elsewhere), max over ranks
    remote = torch.tensor([float((dest != rank).sum())], device=dev)
    dist.all_reduce(remote, op=dist.ReduceOp.MAX)
    nbytes = float(remote) * d * 2
    arena.close()
    arena8.close()
    if rank == 0:
        link = 770.0  # GB/s per direction, measured peer copy on this pool
        floor_us = nbytes / (link * 1e3)
        print(json.dumps({"kernel": "ep_dispatch_combine", "world": W, "tokens_per_rank": tokens, "d": d,
                          "experts": n_experts, "top_k": k, "remote_bytes_per_rank_each_way": int(nbytes),
                          **{k2: round(v, 1) for k2, v in res.items()},
                          "nvlink_floor_us_each_way": round(floor_us, 1),
                          "dispatch_frac_of_link": round(floor_us / res["dispatch_us"], 3),
                          "combine_frac_of_link": round(floor_us / res["combine_us"], 3),
                          "speedup_vs_nccl": round(res["nccl_dispatch_combine_us"] / res["dispatch_combine_us"], 2),
                          "device_error_word": err}))
    dist.destroy_process_group()


def bench_tpgather(M: int = 8192, K: int = 2048, N: int = 8192):
    """Column-parallel linear over the ranks: y[M, N] = all-gather of x @ w_r^T ([M, N / world] per
    rank). Fused: one GEMM whose epilogue stores into every rank's copy (GatherGemm, including its
    flag waits and the copy out of the symmetric buffer). Baseline: the same GEMM, then NCCL
    all_gather_into_tensor and the column interleave. Device time, max over ranks."""
    import torch.distributed as dist

    from astrai_b200.ops._ext import native
    from astrai_b200.parallel.module import GatherGemm

    rank, world = _dist_init()
    C = native()
    hbm, tf, src = peaks()
    n = N // world
    torch.manual_seed(rank)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, K, device="cuda") * 0.05).to(torch.bfloat16)
    gg = GatherGemm()
    loc = torch.empty(M, n, device="cuda", dtype=torch.bfloat16)
    flat = torch.empty(world * M, n, device="cuda", dtype=torch.bfloat16)

    def fused():
        return gg(x, w)

    def gemm_only():
        C.gemm(x, w, loc, None, 0, 0)

    def nccl():
        C.gemm(x, w, loc, None, 0, 0)
        dist.all_gather_into_tensor(flat, loc)
        return flat.view(world, M, n).permute(1, 0, 2).reshape(M, N)

    ref = nccl()
    assert torch.equal(fused(), ref), "fused all-gather GEMM differs from GEMM + NCCL"
    res = {}
    for name, fn in (("fused_ms", fused), ("gemm_only_ms", gemm_only), ("gemm_nccl_ms", nccl)):
        dist.barrier()
        ms = time_fn(fn, warmup=5, iters=20)
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(t.item(), 4)
    torch.cuda.synchronize()
    err = int(C.read_error())
    gg.close()
    dist.barrier()
    if rank == 0:
        fl = 2.0 * M * n * K
        link = 770.0  # measured NVLink peer copy GB/s per direction
        nv_ms = M * n * 2 * (world - 1) / (link * 1e6)
        print(json.dumps({"kernel": "gemm_allgather", "world": world, "M": M, "K": K, "N": N, **res,
                          "speedup_vs_nccl": round(res["gemm_nccl_ms"] / res["fused_ms"], 2),
                          "roofline_ms": round(max(fl / (tf * 1e9), nv_ms), 4),
                          "device_error_word": err}))
    dist.destroy_process_group()


def bench_fsdp_gemm(M: int = 8192, K: int = 2048, N: int = 11264, layers: int = 8):
    """Sharded weights feeding their GEMMs, layer after layer (the FSDP forward): y_l = x @ W_l^T with
    W_l [N, K] (the 1.1B model's packed up|gate weight, 46 MB) held by its owner only.

    Ours (the fused FSDP's path): W_l whole on rank l % world in a symmetric buffer; the copy engines
    pull it over NVLink into one of two local staging buffers on a side stream while the GEMM of layer
    l - 1 runs (no SM time for the transfer). NCCL (torch FSDP2's path): every rank holds 1/world of
    each W_l; all_gather_into_tensor on a side stream, prefetched one layer ahead, then the GEMM.
    Device time per layer, max over ranks; roofline = max(GEMM at the measured burst peak, bytes a
    rank receives per layer over the measured 770 GB/s peer link)."""
    import torch.distributed as dist

    from astrai_b200.ops._ext import native
    from astrai_b200.parallel.symm import SymmetricBuffer

    rank, world = _dist_init()
    C = native()
    hbm, tf, src = peaks()
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(0)
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    wbytes = N * K * 2
    owned = [l for l in range(layers) if l % world == rank]
    pool = SymmetricBuffer(max(1, len(owned)) * wbytes, None, dev, zero=True)
    g = torch.Generator(device=dev).manual_seed(7)
    full = [(torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16) for _ in range(layers)]
    for j, l in enumerate(owned):
        pool.local_view(j * wbytes, wbytes).view(torch.bfloat16).view(N, K).copy_(full[l])
    src_ptr = [pool.ptrs[l % world] + (l // world) * wbytes for l in range(layers)]
    stage = [torch.empty(N, K, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    shard = [f.view(-1).chunk(world)[rank].clone() for f in full]
    gathered = [torch.empty(N * K, device=dev, dtype=torch.bfloat16) for _ in range(2)]
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    side = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    dist.barrier()

    def ours():
        cur = torch.cuda.current_stream()
        ready = [torch.cuda.Event() for _ in range(layers)]
        used = [torch.cuda.Event() for _ in range(layers)]
        for l in range(min(2, layers)):
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                C.peer_copy(stage[l % 2].data_ptr(), src_ptr[l], wbytes)
                ready[l].record(side)
        for l in range(layers):
            cur.wait_event(ready[l])
            C.gemm(x, stage[l % 2], y, None, 0, 0)
            used[l].record(cur)
            if l + 2 < layers:  # refill this buffer for layer l + 2 once the GEMM has read it
                with torch.cuda.stream(side):
                    side.wait_event(used[l])
                    C.peer_copy(stage[l % 2].data_ptr(), src_ptr[l + 2], wbytes)
                    ready[l + 2].record(side)

    def nccl():
        cur = torch.cuda.current_stream()
        ready = [torch.cuda.Event() for _ in range(layers)]
        used = [torch.cuda.Event() for _ in range(layers)]

        def gather(l):
            with torch.cuda.stream(side):
                if l >= 2:
                    side.wait_event(used[l - 2])
                dist.all_gather_into_tensor(gathered[l % 2], shard[l])
                ready[l].record(side)

        side.wait_stream(cur)
        gather(0)
        if layers > 1:
            gather(1)
        for l in range(layers):
            cur.wait_event(ready[l])
            C.gemm(x, gathered[l % 2].view(N, K), y, None, 0, 0)
            used[l].record(cur)
            if l + 2 < layers:
                gather(l + 2)

    def gemm_only():
        for l in range(layers):
            C.gemm(x, full[l], y, None, 0, 0)

    # correctness: the last layer's output of both paths equals the local GEMM
    ref = torch.empty_like(y)
    C.gemm(x, full[-1], ref, None, 0, 0)
    for fn in (ours, nccl):
        fn()
        torch.cuda.synchronize()
        assert torch.equal(y, ref), f"{fn.__name__}: output differs from the local GEMM"
    res = {}
    for name, fn in (("ours_ms", ours), ("nccl_ms", nccl), ("gemm_only_ms", gemm_only)):
        dist.barrier()
        ms = time_fn(fn, warmup=3, iters=10) / layers
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(t.item(), 4)
    torch.cuda.synchronize()
    err = int(C.read_error())
    dist.barrier()
    pool.close()
    if rank == 0:
        fl = 2.0 * M * N * K
        link = 770.0
        nv_ms = wbytes * (world - 1) / world / (link * 1e6)
        roof = max(fl / (tf * 1e9), nv_ms)
        print(json.dumps({"kernel": "fsdp_gather_gemm", "world": world, "M": M, "K": K, "N": N, "layers": layers,
                          **res, "speedup_vs_nccl": round(res["nccl_ms"] / res["ours_ms"], 3),
                          "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / res["ours_ms"], 3),
                          "peak_src": src, "device_error_word": err}))
    dist.destroy_process_group()


def bench_tprow(M: int = 8192, K: int = 8192, N: int = 2048):
    """Row-parallel linear: y[M, N] = sum over ranks of x_r[M, K / world] @ w_r^T. Fused: ReduceGemm
    (GEMM pushing partial rows to their owners as tiles finish, owners sum and broadcast, flag waits,
    copy out). Baseline: the same GEMM, then NCCL all_reduce. Device time, max over ranks."""
    import torch.distributed as dist

    from astrai_b200.ops._ext import native
    from astrai_b200.parallel.module import ReduceGemm

    rank, world = _dist_init()
    C = native()
    _, tf, _ = peaks()
    k = K // world
    torch.manual_seed(rank)
    x = torch.randn(M, k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, k, device="cuda") * 0.05).to(torch.bfloat16)
    rg = ReduceGemm()
    loc = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)

    def gemm_only():
        C.gemm(x, w, loc, None, 0, 0)

    def nccl():
        C.gemm(x, w, loc, None, 0, 0)
        dist.all_reduce(loc)
        return loc

    y = rg(x, w)
    ref = nccl().float()
    err = ((y.float() - ref).norm() / ref.norm()).item()
    res = {}
    for name, fn in (("fused_ms", lambda: rg(x, w)), ("gemm_only_ms", gemm_only), ("gemm_nccl_ms", nccl)):
        dist.barrier()
        ms = time_fn(fn, warmup=5, iters=20)
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(t.item(), 4)
    torch.cuda.synchronize()
    werr = int(C.read_error())
    rg.close()
    dist.barrier()
    if rank == 0:
        fl = 2.0 * M * N * k
        nv_ms = 2 * M * N * 2 * (world - 1) / world / (770.0 * 1e6)
        print(json.dumps({"kernel": "gemm_allreduce", "world": world, "M": M, "K": K, "N": N, **res,
                          "speedup_vs_nccl": round(res["gemm_nccl_ms"] / res["fused_ms"], 2),
                          "roofline_ms": round(max(fl / (tf * 1e9), nv_ms), 4), "rel_err_vs_nccl": round(err, 5),
                          "device_error_word": werr}))
    dist.destroy_process_group()


def bench_skinny():
    """Decode GEMMs (M token rows x weight [N, K]): device time and weight-read bandwidth."""
    from astrai_b200.ops._ext import native

    hbm, tf, src = peaks()
    C = native()
    for M in (1, 4, 16):
        for name, N, K in (("qkv", 3072, 2048), ("o", 2048, 2048), ("upgate", 11264, 2048), ("down", 2048, 5632),
                           ("lm_head", 32000, 2048)):
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            # weights > L2 in total: rotate through 8 copies so every call streams from HBM
            ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) for _ in range(8)]
            y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            it = [0]

            def run():
                C.skinny_gemm(x, ws[it[0] % 8], y, None)
                it[0] += 1
            ms = time_fn(run, warmup=8, iters=40)
            gbs = N * K * 2 / (ms / 1e3) / 1e9
            print(json.dumps({"kernel": "skinny_gemm", "case": name, "M": M, "N": N, "K": K, "us": round(ms * 1e3, 2),
                              "weight_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm, 3), "peak_src": src}))


def bench_sample():
    """Fused sampler on [rows, 32000] logits: greedy, top-k, top-p, both. ``us``: the public
    ``sample()`` per call (host argument handling included); ``kernel_us``: the kernel alone, as the
    decode engine runs it (static argument tensors, 20 calls replayed from one CUDA graph).
    ``ASTRAI_SAMPLE_CTA=0`` times the cluster kernel for every vocabulary."""
    from astrai_b200.inference.sample import _as_row_tensor, _rng_for, fused_sample, sample

    for rows in (1, 4, 32):
        x = torch.randn(rows, 32000, device="cuda") * 3
        for name, kw in (("greedy", dict(temperature=0.0)), ("topk50", dict(temperature=0.8, top_k=50)),
                         ("topp0.95", dict(temperature=0.8, top_p=0.95)),
                         ("topk50_topp0.95", dict(temperature=0.8, top_k=50, top_p=0.95))):
            ms = time_fn(lambda: sample(x, **kw), warmup=5, iters=20)
            args = [_as_row_tensor(kw.get("temperature", 1.0), rows, x.device, torch.float32),
                    _as_row_tensor(kw.get("top_k", 0), rows, x.device, torch.int32),
                    _as_row_tensor(kw.get("top_p", 1.0), rows, x.device, torch.float32),
                    _as_row_tensor(0.0, rows, x.device, torch.float32)]
            tok = torch.empty(rows, dtype=torch.int64, device="cuda")
            lp = torch.empty(rows, dtype=torch.float32, device="cuda")
            rng = _rng_for(x.device)
            fused_sample(x, *args, None, rng, tok, lp)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(20):
                    fused_sample(x, *args, None, rng, tok, lp)
            kern = time_fn(g.replay, warmup=3, iters=10) / 20
            print(json.dumps({"kernel": "sample", "rows": rows, "case": name, "us": round(ms * 1e3, 2),
                              "kernel_us": round(kern * 1e3, 2)}))


def time_flushed(fn, warmup=3, iters=20, flush_bytes=256 << 20):
    """Per-call device time with L2 flushed before every call (a write of ``flush_bytes``, outside
    the timed events): for kernels whose working set would otherwise sit in the 126 MB L2."""
    buf = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        buf.fill_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / iters


def bench_decode():
    """Paged decode attention at the reference's own benchmark shapes
    (csrc/tests/attn_paged_decode_test.cu:280-289: Hq 32, Hkv 4, D 128, page 128) plus batch 32 over
    4096 keys; one query token per row, L2 flushed before every call. Bytes are the K and V rows read
    once (2 x B x Hkv x kv_len x D x 2 bytes). ``ASTRAI_DECODE_TC=0`` times the CUDA-core kernel."""
    from astrai_b200.ops._ext import native

    hbm, _, src = peaks()
    C = native()
    D, Hq, Hkv, page = 128, 32, 4, 128
    for B, L in ((1, 512), (1, 1024), (1, 2048), (1, 4096), (16, 2048), (32, 1024), (32, 4096)):
        n_pages = B * (L // page)
        kc = torch.randn(n_pages, Hkv, page, D, device="cuda").to(torch.bfloat16)
        vc = torch.randn_like(kc)
        table = torch.arange(n_pages, dtype=torch.int32, device="cuda").view(B, L // page)
        lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
        q = torch.randn(B, Hq * D, device="cuda").to(torch.bfloat16)
        out = torch.empty_like(q)
        splits = int(C.decode_splits(B, Hkv, L, 0))
        ws = torch.empty(B * Hq * splits * (D + 2), device="cuda", dtype=torch.float32)
        fn = lambda: C.paged_decode(q, kc, vc, table, lens, out, Hq, D ** -0.5, splits, ws)  # noqa: E731
        ms = time_flushed(fn)
        # back to back without a flush, as the reference's harness times (csrc/tests/test_utils.cuh:37-56)
        warm = time_fn(fn, warmup=10, iters=100)
        # the same, 20 calls replayed from one CUDA graph: device time without the host binding's cost
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(20):
                fn()
        graph = time_fn(g.replay, warmup=3, iters=10) / 20
        nbytes = 2 * B * Hkv * L * D * 2
        if B == 32 and L == 4096:  # the split count against the default heuristic
            sweep = {}
            for sp in (1, 2, 3, 4, 6, 8, 16):
                ws2 = torch.empty(B * Hq * sp * (D + 2), device="cuda", dtype=torch.float32)
                sweep[sp] = round(time_flushed(lambda: C.paged_decode(q, kc, vc, table, lens, out, Hq, D ** -0.5, sp,
                                                                      ws2)) * 1e3, 2)
            print(json.dumps({"kernel": "paged_decode_split_sweep", "B": B, "kv_len": L, "us_by_splits": sweep}))
        print(json.dumps({"kernel": "paged_decode", "impl": "tc" if os.environ.get("ASTRAI_DECODE_TC", "1") != "0"
                          else "cuda_core", "B": B, "Hq": Hq, "Hkv": Hkv, "kv_len": L, "D": D, "page": page,
                          "splits": splits, "us": round(ms * 1e3, 2), "us_warm": round(warm * 1e3, 2),
                          "us_graph": round(graph * 1e3, 2),
                          "GBps": round(nbytes / ms / 1e6, 1),
                          "frac_hbm": round(nbytes / ms / 1e6 / hbm, 3), "peak_src": src}))


def bench_prefill():
    """Prefill attention forward at the reference's own benchmark shapes (csrc/tests/attn_prefill_test.cu
    :12-20: Hq 32, Hkv 4, D 128, q = kv length, causal and not), timed back to back as that harness
    does; SDPA on the same shapes beside it. FLOPs: 4 B Hq q kv D (half when causal)."""
    import torch.nn.functional as F

    from astrai_b200.ops.attention import flash_forward

    _, tf, src = peaks()
    Hq, Hkv, D = 32, 4, 128
    for B, L, causal in ((1, 512, 0), (1, 1024, 0), (1, 2048, 0), (1, 2048, 1), (4, 2048, 1), (1, 4096, 1)):
        q = torch.randn(B * L, Hq * D, device="cuda").to(torch.bfloat16)
        kv = torch.randn(B * L, 2 * Hkv * D, device="cuda").to(torch.bfloat16)
        o = torch.empty_like(q)
        lse = torch.empty(B, Hq, L, device="cuda", dtype=torch.float32)
        fn = lambda: flash_forward(q, 0, kv, 0, kv, Hkv * D, o, lse, B, L, L, Hq, Hkv, D, D ** -0.5,  # noqa: E731
                                   bool(causal), None)
        ms = time_fn(fn, warmup=10, iters=50)
        qt = q.view(B, L, Hq, D).transpose(1, 2)
        kt = kv[:, :Hkv * D].view(B, L, Hkv, D).transpose(1, 2)
        vt = kv[:, Hkv * D:].view(B, L, Hkv, D).transpose(1, 2)
        ms_ref = time_fn(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=bool(causal), enable_gqa=True),
                         warmup=10, iters=50)
        flops = 4.0 * B * Hq * L * L * D * (0.5 if causal else 1.0)
        print(json.dumps({"kernel": "prefill_attention", "B": B, "Hq": Hq, "Hkv": Hkv, "q": L, "kv": L, "D": D,
                          "causal": causal, "ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1),
                          "frac_of_peak": round(flops / ms / 1e9 / tf, 3), "sdpa_ms": round(ms_ref, 4),
                          "peak_src": src}))


def bench_ns():
    """Muon's batched Newton-Schulz chain (5 steps) on the 1.1B model's matrix groups (24 of each),
    with the symmetric-output GEMMs on (``ms_sym``: X X^T and c A A + b A computed on their upper
    triangle, then mirrored) and off."""
    import astrai_b200.optim.fused as F

    _, tf, src = peaks()
    for m, n in ((2048, 11264), (2048, 5632), (2048, 3072), (2048, 2048)):
        X = (torch.randn(24, m, n, device="cuda") / (m * n) ** 0.5).to(torch.bfloat16)
        work = (torch.empty_like(X), torch.empty(24, m, m, device="cuda", dtype=torch.bfloat16),
                torch.empty(24, m, m, device="cuda", dtype=torch.bfloat16))
        res = {}
        for sym in (True, False):
            F.NS_SYM = sym
            res["sym" if sym else "full"] = round(time_fn(lambda: F.newton_schulz_batched(X, 5, work=work),
                                                          warmup=2, iters=5), 3)
        F.NS_SYM = True
        flops = 24 * 5 * (4.0 * m * m * n + 2.0 * m ** 3)
        print(json.dumps({"kernel": "newton_schulz_batched", "batch": 24, "m": m, "n": n, "ms_sym": res["sym"],
                          "ms_full": res["full"], "tflops_full": round(flops / res["full"] / 1e9, 1),
                          "peak_src": src}))


def bench_swiglu_gemm():
    """The up/gate projection with its SwiGLU: the plain GEMM writing h = (u, g) and the separate
    SwiGLU kernel, against the SwiGLU-epilogue GEMM writing h and a (training) or only a (no
    autograd); at a 2048-token prefill of d 1536 / FFN 6912 and the 1.1B step's 8192 x 2048 / 5632.
    Warm (back to back) and with L2 flushed before every call, us per call."""
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.activation import swiglu

    C = native()
    for M, d, F in ((2048, 1536, 6912), (8192, 2048, 5632)):
        x = torch.randn(M, d, device="cuda").to(torch.bfloat16)
        w = (torch.randn(2 * F, d, device="cuda") * 0.02).to(torch.bfloat16)
        h = torch.empty(M, 2 * F, device="cuda", dtype=torch.bfloat16)
        a = torch.empty(M, F, device="cuda", dtype=torch.bfloat16)
        fns = {"gemm": lambda: C.gemm(x, w, h, None, 0, 0, 1.0, 0.0, 0),
               "swiglu_kernel": lambda: swiglu(h),
               "fused_h_and_a": lambda: C.gemm_swiglu(1, x, w, h, a, None),
               "fused_a_only": lambda: C.gemm_swiglu(1, x, w, None, a, None)}
        res = {k: [round(time_fn(f, 5, 30) * 1e3, 1), round(time_flushed(f, 3, 20) * 1e3, 1)] for k, f in fns.items()}
        print(json.dumps({"kernel": "gemm_swiglu", "M": M, "d": d, "F": F, "us_warm_flushed": res}))


def bench_rope_gemm():
    """The QKV projection with RoPE: the plain GEMM followed by the in-place RoPE kernel, against the
    GEMM with RoPE on its q and k columns in the epilogue; at the 1.1B step's shape (8192 x 2048 ->
    3072, 20 rotated heads of 128) and a 2048-token prefill of the reference benchmark's model
    (2048 x 1536 -> 2048, 28 rotated heads of 64). Warm and L2 flushed, us per call."""
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.rope import rope_inplace, rope_table

    C = native()
    for M, d, N, hd, heads, seq in ((8192, 2048, 3072, 128, 20, 2048), (2048, 1536, 2048, 64, 28, 512)):
        x = torch.randn(M, d, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, d, device="cuda") * 0.02).to(torch.bfloat16)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        tab = rope_table(hd, 4096, 1e6, device="cuda")

        def separate():
            C.gemm(x, w, y, None, 0, 0, 1.0, 0.0, 0)
            rope_inplace(y, 0, heads, hd, tab, None, seq)

        fns = {"gemm_then_rope": separate,
               "gemm_rope_epilogue": lambda: C.gemm_rope(x, w, y, tab, None, seq, heads * hd, hd)}
        res = {k: [round(time_fn(f, 5, 30) * 1e3, 1), round(time_flushed(f, 3, 20) * 1e3, 1)] for k, f in fns.items()}
        print(json.dumps({"kernel": "gemm_rope", "M": M, "K": d, "N": N, "head_dim": hd, "us_warm_flushed": res}))


def bench_gemm_shapes():
    """Tile plans on the GEMMs of a 2048-token prefill (d 1536, 24/4 heads of 64, FFN 6912, vocab
    10000) and of the 1.1B step, L2 flushed before every call (us): automatic plan (0), CTA pairs
    unsplit (1024), pairs with the last-wave split (1026), pairs with every k-block split (1027),
    single CTA 128 x 256 (256), 256 x 192 pair tiles (192, K-major B only), cuBLAS."""
    from astrai_b200.ops._ext import native

    C = native()
    shapes = [(2048, 2048, 1536, "qkv"), (2048, 1536, 1536, "o"), (2048, 13824, 1536, "upgate"),
              (2048, 1536, 6912, "down"), (2048, 10000, 1536, "lm_head"), (8192, 3072, 2048, "step_qkv"),
              (8192, 2048, 2048, "step_o"), (8192, 11264, 2048, "step_upgate"), (8192, 2048, 5632, "step_down"),
              (8192, 32000, 2048, "step_lm_head")]
    # the step's weight gradients dW = dY^T X: both operands MN-major ([tokens][out], [tokens][in])
    wgrad = [(3072, 2048, 8192, "wgrad_qkv"), (2048, 2048, 8192, "wgrad_o"), (11264, 2048, 8192, "wgrad_upgate"),
             (2048, 5632, 8192, "wgrad_down")]
    # data gradients dX = dY W: B = W stored [out][in] = [K][N], MN-major
    dgrad = [(8192, 2048, 11264, "dgrad_upgate"), (8192, 2048, 32000, "dgrad_lm_head"), (8192, 5632, 2048, "dgrad_down")]
    for M, N, K, name in shapes + wgrad + dgrad:
        amn, bmn = int(name.startswith("wgrad")), int(name.startswith(("wgrad", "dgrad")))
        a = torch.randn((K, M) if amn else (M, K), device="cuda").to(torch.bfloat16)
        b = torch.randn((K, N) if bmn else (N, K), device="cuda").to(torch.bfloat16)
        d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        res = {}
        for fb in (0, 1024, 1026, 1027, 256) + (() if bmn else (192,)):
            res[str(fb)] = round(time_flushed(lambda: C.gemm(a, b, d, None, amn, bmn, 1.0, 0.0, fb), 3, 20) * 1e3, 1)
        res["cublas"] = round(time_flushed(lambda: torch.matmul(a.t() if amn else a, b if bmn else b.t()), 3, 20)
                              * 1e3, 1)
        print(json.dumps({"kernel": "gemm", "case": name, "M": M, "N": N, "K": K, "us": res}))


def bench_elementwise():
    """SwiGLU forward / backward and in-place RoPE at the 1.1B step's shapes (8192 rows; FFN 5632;
    q and k heads 16 + 4 of 128 in the 3072-wide QKV output), L2 flushed before every call; bytes
    are the algorithmic reads + writes."""
    from astrai_b200.ops._ext import native
    from astrai_b200.ops.rope import rope_inplace, rope_table

    hbm, _, src = peaks()
    C = native()
    rows, Fw = 8192, 5632
    h = torch.randn(rows, 2 * Fw, device="cuda").to(torch.bfloat16)
    a = torch.empty(rows, Fw, device="cuda", dtype=torch.bfloat16)
    da = torch.randn(rows, Fw, device="cuda").to(torch.bfloat16)
    dh = torch.empty_like(h)
    qkv = torch.randn(rows, 24 * 128, device="cuda").to(torch.bfloat16)
    tab = rope_table(128, 2048, 1e6, device="cuda")
    cases = [("swiglu_fwd", lambda: C.swiglu_fwd(h, a), rows * Fw * 2 * 3),
             ("swiglu_bwd", lambda: C.swiglu_bwd(da, h, dh), rows * Fw * 2 * 5),
             ("rope", lambda: rope_inplace(qkv, 0, 20, 128, tab, None, 2048), rows * 20 * 128 * 2 * 2)]
    for name, fn, nbytes in cases:
        us = time_flushed(fn, 3, 20) * 1e3
        print(json.dumps({"kernel": name, "us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                          "frac_of_hbm": round(nbytes / us / 1e3 / hbm, 3), "peak_src": src}))


def bench_norm(rows: int = 8192, D: int = 2048):
    """RMSNorm forward, backward and the fork backward (residual-branch gradient added) at the 1.1B
    step's shape; bytes are the algorithmic reads + writes (bf16 rows, fp32 rstd)."""
    from astrai_b200.ops._ext import native

    hbm, _, src = peaks()
    C = native()
    x = torch.randn(rows, D, device="cuda", dtype=torch.bfloat16)
    dy, dres = torch.randn_like(x), torch.randn_like(x)
    w = (1 + 0.1 * torch.randn(D, device="cuda")).to(torch.bfloat16)
    y, dx = torch.empty_like(x), torch.empty_like(x)
    rstd = torch.empty(rows, device="cuda", dtype=torch.float32)
    dw = torch.empty(D, device="cuda", dtype=torch.bfloat16)
    scratch = torch.empty(C.rmsnorm_bwd_scratch(rows, D), device="cuda", dtype=torch.float32)
    row = rows * D * 2
    cases = [("rmsnorm_fwd", lambda: C.rmsnorm_fwd(x, w, y, rstd, 1e-5), 2 * row + rows * 4),
             ("rmsnorm_bwd", lambda: C.rmsnorm_bwd(dy, x, w, rstd, dx, dw, scratch), 3 * row + rows * 4),
             ("rmsnorm_bwd_fork", lambda: C.rmsnorm_bwd(dy, x, w, rstd, dx, dw, scratch, dres), 4 * row + rows * 4)]
    for name, fn, nbytes in cases:
        ms = time_fn(fn, warmup=5, iters=50)
        gbs = nbytes / ms / 1e6
        print(json.dumps({"kernel": name, "rows": rows, "D": D, "us": round(ms * 1e3, 2), "GB/s": round(gbs, 1),
                          "frac_of_hbm": round(gbs / hbm, 3), "peak_src": src}))


def main(argv=None):
    args = argv or sys.argv[1:] or ["all"]
    which = args[0]
    torch.manual_seed(0)
    if which == "allreduce":
        bench_allreduce()
        return
    if which == "ep":
        bench_ep()
        return
    if which == "tpgather":
        bench_tpgather()
        return
    if which == "tprow":
        bench_tprow()
        return
    if which == "fsdp":
        bench_fsdp_gemm()
        return
    if which in ("skinny", "all"):
        bench_skinny()
    if which in ("sample", "all"):
        bench_sample()
    if which in ("decode", "all"):
        bench_decode()
    if which in ("prefill", "all"):
        bench_prefill()
    if which in ("ns", "all"):
        bench_ns()
    if which in ("elementwise", "all"):
        bench_elementwise()
    if which in ("swiglu_gemm", "all"):
        bench_swiglu_gemm()
    if which in ("rope_gemm", "all"):
        bench_rope_gemm()
    if which in ("gemm_shapes", "all"):
        bench_gemm_shapes()
    if which in ("gemm", "all"):
        bench_gemm(args[1] if which == "gemm" and len(args) > 1 else None)
    if which in ("norm", "all"):
        bench_norm()
    if which in ("attn", "all"):
        try:
            from astrai_b200.ops.attention import bench_attention

            bench_attention(time_fn, peaks)
        except ImportError:
            pass


if __name__ == "__main__":
    main()
