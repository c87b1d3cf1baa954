"""Kernel-time breakdown of one training step (torch profiler / CUPTI, CUDA activity only).

    python -m nuvla_forge_b200.bench.step_profile --model-config 1b --batch-size 8

Runs two warm-up steps, then records one optimizer step of one micro-batch and
prints device time by category (GEMM, attention, native kernels, other) and
the top kernels. Times taken under a profiler are for shares, not benchmarks.
"""

from __future__ import annotations

import argparse

import torch


NATIVE_GEMM = ("gemm_pair_kernel", "gemm_small_kernel", "tc_kernel", "ag_gemm")
NATIVE_ATTN = ("attn_fwd", "attn_bwd", "attn_pre", "attn_dq")


def category(name: str) -> str:
    """Kernel class: native (this library's) or library GEMM / attention, other native, other."""
    n = name.lower()
    if any(k in n for k in NATIVE_GEMM):
        return "native gemm"
    if any(k in n for k in NATIVE_ATTN):
        return "native attention"
    if "nfb::" in n or n.startswith("nfb") or "adamw_kernel" in n:
        return "native other"
    if "sdpa" in n or "flash" in n or "fmha" in n or "attention" in n:
        return "library attention"
    if "nvjet" in n or "gemm" in n or "cutlass" in n or "xmma" in n or "cublas" in n:
        return "library gemm"
    return "other"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-config", default="1b")
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--top", type=int, default=40)
    args = ap.parse_args(argv)
    from torch.profiler import ProfilerActivity, profile

    from ..data import SampleSpec, SyntheticBatchSource
    from ..models import NuVLAConfig
    from ..parallel.dist import setup_distributed
    from ..train import Trainer

    info = setup_distributed()
    cfg = NuVLAConfig.preset(args.model_config)
    tr = Trainer(cfg, info, grad_accum=1, bf16=True)
    src = SyntheticBatchSource(SampleSpec.for_model(cfg), args.batch_size, pin=False)
    batch = [tr.to_device(src.batch(0))]
    for _ in range(2):
        tr.step(batch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        e0.record()
        tr.step(batch)
        e1.record()
        torch.cuda.synchronize()
    elapsed_ms = e0.elapsed_time(e1)
    rows = sorted((e for e in prof.key_averages() if e.device_time_total > 0), key=lambda e: -e.device_time_total)
    total = sum(e.device_time_total for e in rows)
    cats: dict[str, float] = {}
    for e in rows:
        cats[category(e.key)] = cats.get(category(e.key), 0.0) + e.device_time_total
    print(f"model {args.model_config}, micro-batch {args.batch_size}: total device time {total / 1e3:.1f} ms "
          f"in {elapsed_ms:.1f} ms elapsed (kernels busy {100 * total / 1e3 / elapsed_ms:.1f}% of the step; "
          f"below 100% = the GPU waited on the host or on dependencies)")
    for c, v in sorted(cats.items(), key=lambda kv: -kv[1]):
        print(f"  {c:10s} {v / 1e3:9.2f} ms  {100 * v / total:5.1f}%")
    for e in rows[: args.top]:
        print(f"{e.device_time_total / 1e3:9.2f} ms {e.count:6d}  {100 * e.device_time_total / total:5.1f}%  {e.key[:110]}")


if __name__ == "__main__":
    main()
