"""Device-timed micro-benchmarks of the framework's kernels.

    python -m astrai_b200.utils.kernel_bench [gemm|attn|decode|sample|all]
    torchrun --nproc-per-node N -m astrai_b200.utils.kernel_bench allreduce

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


def bench_gemm():
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
        ("square_8192", 8192, 8192, 8192, 0, 0),
    ]
    for name, M, N, K, amn, bmn in cases:
        a = torch.randn((K, M) if amn else (M, K), device="cuda", dtype=torch.bfloat16)
        b = torch.randn((K, N) if bmn else (N, K), device="cuda", dtype=torch.bfloat16)
        d = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = time_fn(lambda: C.gemm(a, b, d, None, amn, bmn, 1.0, 0.0, 0))
        A = a.t() if amn else a
        B = b if bmn else b.t()
        ms_ref = time_fn(lambda: torch.matmul(A, B))
        fl = 2.0 * M * N * K
        print(json.dumps({"kernel": "gemm", "case": name, "M": M, "N": N, "K": K, "ms": round(ms, 4),
                          "tflops": round(fl / ms / 1e9, 1), "frac_of_peak": round(fl / ms / 1e9 / tf, 3),
                          "peak_src": src, "cublas_ms": round(ms_ref, 4),
                          "cublas_tflops": round(fl / ms_ref / 1e9, 1)}))


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
    """Fused sampler on [rows, 32000] logits: greedy, top-k, top-p, both."""
    from astrai_b200.inference.sample import sample

    for rows in (1, 4, 32):
        x = torch.randn(rows, 32000, device="cuda") * 3
        for name, kw in (("greedy", dict(temperature=0.0)), ("topk50", dict(temperature=0.8, top_k=50)),
                         ("topp0.95", dict(temperature=0.8, top_p=0.95)),
                         ("topk50_topp0.95", dict(temperature=0.8, top_k=50, top_p=0.95))):
            ms = time_fn(lambda: sample(x, **kw), warmup=5, iters=20)
            print(json.dumps({"kernel": "sample", "rows": rows, "case": name, "us": round(ms * 1e3, 2)}))


def main(argv=None):
    which = (argv or sys.argv[1:] or ["all"])[0]
    torch.manual_seed(0)
    if which == "allreduce":
        bench_allreduce()
        return
    if which in ("skinny", "all"):
        bench_skinny()
    if which in ("sample", "all"):
        bench_sample()
    if which in ("gemm", "all"):
        bench_gemm()
    if which in ("attn", "all"):
        try:
            from astrai_b200.ops.attention import bench_attention

            bench_attention(time_fn, peaks)
        except ImportError:
            pass


if __name__ == "__main__":
    main()
