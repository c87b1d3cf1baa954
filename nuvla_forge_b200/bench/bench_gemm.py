"""Linear-layer GEMMs: the CTA-pair tcgen05 kernel (csrc/gemm.cu) vs cuBLAS (torch.matmul).

    python -m nuvla_forge_b200.bench.bench_gemm [--out reports/gemm.json] [--quick]

Shapes are the linear layers of one BASELINE config-3 micro-batch (8 samples): the ViT
(98304 tokens, d 1024, MLP 4096), the backbone (27136 tokens, d 2048, GQA qkv 4096, SwiGLU
5632) and the DiT context projection, plus the 8192^3 square GEMM. Each shape is timed in its
three roles: forward Y = X W^T, input gradient dX = dY W and weight gradient dW = dY^T X
(fp32 output, as the trainer accumulates it). Time = median of CUDA-event timings with L2
flushed (256 MB write) between iterations; TF/s = 2 M N K / time.
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from ..profiling import load_measured_peaks

SHAPES = [  # name, tokens M, out N, in K
    ("square 8192^3", 8192, 8192, 8192),
    ("vit qkv", 98304, 3072, 1024),
    ("vit proj", 98304, 1024, 1024),
    ("vit mlp up", 98304, 8192, 1024),
    ("vit mlp down", 98304, 1024, 4096),
    ("backbone qkv", 27136, 4096, 2048),
    ("backbone proj", 27136, 2048, 2048),
    ("backbone gate_up", 27136, 11264, 2048),
    ("backbone down", 27136, 2048, 5632),
    ("dit ctx kv", 27136, 2048, 2048),
]


def _time(fn, iters, flush):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def sustained(seconds: float, out_path: str | None) -> None:
    """Back-to-back GEMMs for ``seconds`` per implementation and role, with SM clock and power sampled:
    under the 1 kW cap the sustained rate depends on energy per FLOP, not only on burst speed."""
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
    from bench import ClockSampler, visible_gpu_ids

    from ..ops import linear as L

    rows = []
    for name, M, N, K in (SHAPES[0], SHAPES[1], SHAPES[3]):
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
        w = torch.randn(N, K, generator=g, device="cuda").to(torch.bfloat16)
        dy = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        dx = torch.empty(M, K, dtype=torch.bfloat16, device="cuda")
        dw = torch.zeros(N, K, dtype=torch.float32, device="cuda")
        dwb = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
        roles = [("fwd", lambda: L.gemm(x, w, out=y), lambda: torch.mm(x, w.t(), out=y)),
                 ("dgrad", lambda: L.gemm(dy, w, b_mn=True, out=dx), lambda: torch.mm(dy, w, out=dx)),
                 ("wgrad", lambda: L.gemm_acc(dy, x, dw, a_mn=True, b_mn=True, accumulate=True),
                  lambda: torch.mm(dy.t(), x, out=dwb))]
        for role, nat_fn, ref_fn in roles:
            for impl, fn in (("native", nat_fn), ("cublas", ref_fn)):
                for _ in range(5):
                    fn()
                torch.cuda.synchronize()
                one = _time(fn, 3, torch.empty(1, device="cuda"))
                n = max(1, int(seconds * 1e3 / one))
                smp = ClockSampler(visible_gpu_ids())
                smp.start()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(n):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                clk = smp.stop()
                ms = e0.elapsed_time(e1) / n
                tf = 2.0 * M * N * K / ms / 1e9
                row = {"shape": name, "role": role, "impl": impl, "iters": n, "ms": ms, "tflops": tf, "clocks": clk,
                       "pj_per_flop": (clk.get("power_w") or 0) / (tf * 1e12) * 1e12 if tf else None}
                rows.append(row)
                print(f"sustained {name:14s} {role:6s} {impl:6s} {tf:7.1f} TF/s  sm {clk.get('sm_mhz')} MHz "
                      f"power {clk.get('power_w')} W  {row['pj_per_flop']:.3f} pJ/FLOP", flush=True)
        del x, w, dy, y, dx, dw, dwb
        torch.cuda.empty_cache()
    if out_path:
        Path(out_path).write_text(json.dumps({"sustained_s": seconds, "rows": rows}, indent=1))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="reports/gemm.json")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--quick", action="store_true", help="first three shapes only")
    ap.add_argument("--sustained", type=float, default=0.0,
                    help="instead: run each implementation back to back for this many seconds (clock/power)")
    args = ap.parse_args(argv)
    if args.sustained > 0:
        sustained(args.sustained, args.out)
        return
    from ..ops import linear as L

    peaks = load_measured_peaks()
    peak = peaks.get("bf16_tflops") if peaks else None
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")
    rows = []
    shapes = SHAPES[:3] if args.quick else SHAPES
    for name, M, N, K in shapes:
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
        w = torch.randn(N, K, generator=g, device="cuda").to(torch.bfloat16)
        dy = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
        dw = torch.empty(N, K, dtype=torch.float32, device="cuda")
        flops = 2.0 * M * N * K
        roles = {
            "fwd": (lambda: L.gemm(x, w), lambda: torch.matmul(x, w.t())),
            "dgrad": (lambda: L.input_grad(dy, w), lambda: torch.matmul(dy, w)),
            "wgrad": (lambda: L.gemm_acc(dy, x, dw, a_mn=True, b_mn=True), lambda: torch.mm(dy.t(), x).float()),
        }
        for role, (ours, ref) in roles.items():
            t_ours = _time(ours, args.iters, flush)
            t_ref = _time(ref, args.iters, flush)
            torch.cuda.synchronize()
            L.check_status()
            row = {"shape": name, "role": role, "M": M, "N": N, "K": K,
                   "native_ms": t_ours, "cublas_ms": t_ref,
                   "native_tflops": flops / t_ours / 1e9, "cublas_tflops": flops / t_ref / 1e9,
                   "speedup": t_ref / t_ours}
            if peak:
                row["native_frac_of_measured_peak"] = row["native_tflops"] / peak
            rows.append(row)
            print(f"{name:18s} {role:6s} native {t_ours:8.3f} ms {row['native_tflops']:7.1f} TF/s | "
                  f"cublas {t_ref:8.3f} ms {row['cublas_tflops']:7.1f} TF/s | x{row['speedup']:.3f}", flush=True)
        del x, w, dy, dw
        torch.cuda.empty_cache()
    out = {"measured_peaks": peaks, "rows": rows,
           "note": "cuBLAS wgrad = bf16 mm then fp32 cast (what autograd + fp32 accumulation would cost)"}
    if args.out:
        Path(args.out).parent.mkdir(parents=True, exist_ok=True)
        Path(args.out).write_text(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
