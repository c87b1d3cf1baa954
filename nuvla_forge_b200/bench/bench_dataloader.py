"""Data-loading throughput, isolated and in situ.

    python -m nuvla_forge_b200.bench.bench_dataloader [--model-config ref] [--batches 50]

Parity: nuvla_forge/bench/bench_dataloader.py — loader-only samples/s for
four loader configurations (naive 2 workers; tuned 8 workers pinned; tuned +
CUDA prefetch; 16 workers) and the GPU idle fraction with a real fwd+bwd per
batch. Added: the native pinned ``SyntheticBatchSource`` as a fifth row.
"""

from __future__ import annotations

import argparse
import json
import time
from pathlib import Path

import torch

from ..data import (CudaPrefetcher, LoaderConfig, SampleSpec, SyntheticBatchSource, build_dataset,
                    build_fast_loader, build_naive_loader, describe_environment)
from ..models import NuVLA, NuVLAConfig


def measure_loader(loader, n_batches, device, prefetch=False):
    """Loader-only samples/s (no compute between batches); 5 warm-up batches."""
    if prefetch and device.type == "cuda":
        loader = CudaPrefetcher(loader, device)
    it = iter(loader)
    for _ in range(5):
        next(it, None)
    if device.type == "cuda":
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    seen = 0
    for _ in range(n_batches):
        b = next(it, None)
        if b is None:
            break
        seen += b["images"].shape[0]
    if device.type == "cuda":
        torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    return {"samples_per_sec": seen / dt, "batches": n_batches, "seconds": dt}


def measure_idle(loader, device, cfg, n_batches=30, prefetch=False):
    """GPU idle % = 1 - (device-busy time of fwd+bwd) / wall time, after 5 warm-up batches."""
    model = NuVLA(cfg).to(device, torch.bfloat16)
    if prefetch and device.type == "cuda":
        loader = CudaPrefetcher(loader, device)
    it = iter(loader)
    busy, wall0 = 0.0, None
    for i in range(n_batches):
        b = next(it, None)
        if b is None:
            break
        b = {k: v.to(device, non_blocking=True) for k, v in b.items() if isinstance(v, torch.Tensor)}
        if i == 5:
            torch.cuda.synchronize()
            wall0, busy = time.perf_counter(), 0.0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        out = model(b["images"], b["trajectory"], b["text_tokens"], b["text_targets"])
        out["loss"].backward()
        e1.record()
        torch.cuda.synchronize()
        if wall0 is not None:
            busy += e0.elapsed_time(e1)
    wall = (time.perf_counter() - wall0) * 1e3
    return {"wall_ms": wall, "gpu_busy_ms": busy, "gpu_idle_pct": 100.0 * (1 - busy / wall)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--dataset", default="synthetic")
    ap.add_argument("--data-root", default=None)
    ap.add_argument("--model-config", default="ref")
    ap.add_argument("--batch-size", type=int, default=8)
    ap.add_argument("--batches", type=int, default=50)
    ap.add_argument("--out", default="reports/dataloader.json")
    args = ap.parse_args(argv)
    device = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    cfg = NuVLAConfig.preset(args.model_config)
    spec = SampleSpec.for_model(cfg)
    kw = {"spec": spec}
    if args.data_root:
        kw["root"] = args.data_root
    ds = build_dataset(args.dataset, **kw)
    env = describe_environment()
    print(f"dataset {args.dataset}: {len(ds)} samples | env {env}")
    report = {"dataset": args.dataset, "model": args.model_config, "env": env, "configs": []}
    configs = [("naive (2 workers, no pin)", build_naive_loader, {"num_workers": 2}, False),
               ("tuned (8 workers, pinned)", build_fast_loader, {"num_workers": 8, "prefetch_factor": 4}, False),
               ("tuned + cuda prefetch", build_fast_loader, {"num_workers": 8, "prefetch_factor": 4}, True),
               ("tuned + 16 workers", build_fast_loader, {"num_workers": 16, "prefetch_factor": 6}, True)]
    print(f"{'config':<34} {'samples/s':>11} {'gpu idle':>10}")
    for name, build, over, prefetch in configs:
        lcfg = LoaderConfig(batch_size=args.batch_size, max_text_len=cfg.max_text_len, **over)
        try:
            thr = measure_loader(build(ds, lcfg), args.batches, device, prefetch)
            idle = (measure_idle(build(ds, lcfg), device, cfg, prefetch=prefetch) if device.type == "cuda"
                    else {"gpu_idle_pct": float("nan")})
            row = dict(config=name, **thr, **idle)
        except Exception as exc:  # noqa: BLE001 - one config failing is that config's result
            row = {"config": name, "error": str(exc)}
        report["configs"].append(row)
        print(f"{name:<34} {row.get('samples_per_sec', float('nan')):11.1f} {row.get('gpu_idle_pct', float('nan')):9.1f}%")
    if args.dataset == "synthetic":
        src = SyntheticBatchSource(spec, args.batch_size, n_batches=args.batches + 5)
        thr = measure_loader(src, args.batches, device, prefetch=device.type == "cuda")
        row = dict(config="native pinned synthetic source", **thr)
        report["configs"].append(row)
        print(f"{row['config']:<34} {row['samples_per_sec']:11.1f}")
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(report, indent=2))
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
