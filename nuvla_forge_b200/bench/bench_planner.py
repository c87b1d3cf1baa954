"""Planning latency: the eager DiT sampler vs the CUDA-graph planner (nuvla_forge_b200.serve).

    python -m nuvla_forge_b200.bench.bench_planner [--model-config 1b] [--steps 10]

For batch sizes 1, 8 and 32 at the given config: the context is computed once;
the timed part is ``steps`` Euler steps of the DiT (CUDA events, median of 20).
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from ..models import NuVLA, NuVLAConfig
from ..serve import GraphedPlanner


def _time(fn, iters=20):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-config", default="1b")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--out", default="reports/planner.json")
    args = ap.parse_args(argv)
    cfg = NuVLAConfig.preset(args.model_config)
    model = NuVLA(cfg).cuda().to(torch.bfloat16).eval()
    ctx_len = cfg.n_images * cfg.pooled_tokens + cfg.text_len if cfg.backbone_over_images else 32
    d = cfg.t_dim if cfg.backbone_over_images else cfg.vision_dim
    rows = []
    for bs in (1, 8, 32):
        ctx = torch.randn(bs, ctx_len, d, device="cuda").to(torch.bfloat16)
        eager = _time(lambda: model.dit.sample(ctx, args.steps))
        planner = GraphedPlanner(model, bs, ctx_len, args.steps)
        graphed = _time(lambda: planner(ctx))
        rows.append({"batch": bs, "eager_ms": eager, "graphed_ms": graphed, "speedup": eager / graphed})
        print(f"batch {bs:3d}: eager {eager:7.2f} ms | graphed {graphed:7.2f} ms | {eager / graphed:.2f}x")
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps({"model": args.model_config, "steps": args.steps, "rows": rows}, indent=2))


if __name__ == "__main__":
    main()
