"""Per-kernel share of one training step (torch.profiler / CUPTI activity records).

    python -m astrai_b200.utils.step_profile [--model dense|moe] [--accum 8] [--top 30] [--json out.json]

Builds the benchmark's model (dense 1.1B: 24 L, d 2048, 16/4 heads, FFN
5632, vocab 32000, batch 4 x seq 2048; or the MoE config), runs two warm-up
optimizer steps, then records one step and prints every kernel's device time,
call count and share of the step's kernel time, plus the share per category
(GEMM, attention fwd/bwd, norm, loss, optimizer, ...). Shares only: times
under a profiler are not benchmark numbers.
"""

from __future__ import annotations

import argparse
import json
from collections import defaultdict

import torch

DENSE = dict(vocab_size=32000, hidden_size=2048, num_hidden_layers=24, rms_norm_eps=1e-5, intermediate_size=5632,
             tie_word_embeddings=False, max_position_embeddings=2048, rope_theta=1e6, num_attention_heads=16,
             num_key_value_heads=4)
MOE = dict(DENSE, num_hidden_layers=16, max_position_embeddings=4096, ffn_type="moe", n_routed_experts=64,
           n_shared_experts=2, n_activated_experts=6, moe_intermediate_size=1408, first_k_dense=1,
           moe_aux_loss_coef=0.01)

CATEGORIES = (("gemm", ("gemm_kernel", "gemm", "cutlass", "sm100_xmma", "nvjet")),
              ("attn_fwd", ("flash_fwd",)), ("attn_bwd", ("flash_bwd", "flash_dq")),
              ("norm", ("rmsnorm", "reduce_cols")), ("loss", ("ce_fwd", "ce_bwd")),
              ("optimizer", ("adamw", "muon", "sumsq", "clip_coef")),
              ("moe", ("moe_router", "ep_")), ("elementwise", ("rope", "swiglu", "embedding", "f32_to_bf16",
                                                               "transpose")),
              ("comm", ("allreduce", "nccl")))


def category(name: str) -> str:
    low = name.lower()
    for cat, keys in CATEGORIES:
        if any(k in low for k in keys):
            return cat
    return "other"


def main(argv=None) -> None:
    from torch.profiler import ProfilerActivity, profile

    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.ops.loss import cross_entropy
    from astrai_b200.optim import MuonMix, clip_grad_norm_

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--model", default="dense", choices=["dense", "moe"])
    p.add_argument("--accum", type=int, default=None)
    p.add_argument("--top", type=int, default=30)
    p.add_argument("--json", type=str, default=None)
    a = p.parse_args(argv)
    cfg, (B, S, acc) = (DENSE, (4, 2048, 8)) if a.model == "dense" else (MOE, (2, 4096, 1))
    acc = a.accum or acc
    torch.manual_seed(0)
    dev = torch.device("cuda")
    with dev:
        model = AutoRegressiveLM(AutoRegressiveLMConfig(**cfg)).to(torch.bfloat16)
    opt = MuonMix(model, lr=0.02, weight_decay=0.1, adamw_lr=1e-4, adamw_weight_decay=0.1,
                  adjust_lr_fn="match_rms_adamw")
    data = torch.randint(0, cfg["vocab_size"], (acc, B, S + 1), device=dev)

    def step():
        for m in range(acc):
            out = model(data[m, :, :-1])
            loss = cross_entropy(out["logits"], data[m, :, 1:])
            if "aux_loss" in out:
                loss = loss + out["aux_loss"]
            (loss / acc).backward()
        clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    per = defaultdict(lambda: [0.0, 0])
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            per[ev.name][0] += ev.time_range.elapsed_us() / 1e3  # kernel records: start/end on the device
            per[ev.name][1] += 1
    total = sum(v[0] for v in per.values()) or 1.0
    cats = defaultdict(float)
    for n, (ms, _) in per.items():
        cats[category(n)] += ms
    rows = sorted(per.items(), key=lambda kv: -kv[1][0])
    print(f"step kernel time {total:.1f} ms ({a.model}, {acc} x {B} x {S} tokens)")
    for cat, ms in sorted(cats.items(), key=lambda kv: -kv[1]):
        print(f"  {cat:12s} {ms:9.2f} ms  {100 * ms / total:5.1f} %")
    for n, (ms, c) in rows[:a.top]:
        print(f"  {ms:9.2f} ms {100 * ms / total:5.1f} % x{c:5d}  {n[:110]}")
    if a.json:
        with open(a.json, "w") as fh:
            json.dump({"total_ms": total, "categories": cats,
                       "kernels": [{"name": n, "ms": ms, "calls": c} for n, (ms, c) in rows]}, fh, indent=1)


if __name__ == "__main__":
    main()
