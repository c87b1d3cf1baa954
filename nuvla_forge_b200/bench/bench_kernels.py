"""Kernel microbenchmarks (BASELINE config 2 plus the reference's own sweep shapes).

    python -m nuvla_forge_b200.bench.bench_kernels [--out reports/kernels.json] [--quick]

Parity: nuvla_forge/bench/bench_kernels.py (timeit with CUDA events, eager vs
fused, achieved GB/s and a roofline note). Differences: the roofline
denominators are the MEASURED peaks (MEASURED_PEAKS.json: STREAM-style copy
GB/s and cuBLAS bf16 TFLOP/s), not a spec-sheet table; each case also times
the reference's own Triton kernel when the reference is installed in
baseline/_ref; between timed iterations a 256 MiB buffer is written to flush
the 126 MB L2 (or the inputs are larger than L2, noted per case).

Byte counts are the algorithmic minimum of each op:
  adaLN fwd+bwd: read x, y; write h, out; read dh, dout, h, y; write dx, dy = 10 tensors
  SwiGLU fwd+bwd: read a, b; write out; read dout, a, b; write da, db = 8 tensors
  CE fwd+bwd: FLOPs of 3 GEMMs of 2*M*H*V each (logits, dW, dh)
  patchify: read the uint8 frames, write the bf16 patch rows (the reference normalises whole frames
    in eager PyTorch and cuts patches inside its Conv2d; "eager" here is that normalisation plus
    the unfold into patch rows)
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

from ..ops import chunked_cross_entropy, fused_adaln_residual_rmsnorm, fused_swiglu
from ..ops.reference import adaln_residual_rmsnorm_ref, chunked_cross_entropy_ref, swiglu_ref
from ..profiling import bandwidth_gb_s, load_measured_peaks, roofline_note, tflops

_FLUSH = None


def flush_l2():
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")
    _FLUSH.zero_()


def timeit(fn, iters=20, warmup=5, flush=True):
    """Median CUDA-event time of fn (ms), L2 flushed before each timed call."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    return times[len(times) // 2]


def timeit_device(fn, iters=20, warmup=5):
    """Median CUDA-event time of fn's GPU work alone (ms): L2 flushed, then a ~0.1 ms device sleep
    queued before the start event so the host's launch overhead overlaps it."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush_l2()
        torch.cuda._sleep(200_000)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    return times[len(times) // 2]


def reference_kernels():
    """The reference's Triton kernels (unmodified, baseline/_ref), or None."""
    root = Path(__file__).resolve().parents[2] / "baseline" / "_ref"
    if not (root / "nuvla_forge").is_dir():
        return None
    sys.path.insert(0, str(root))
    try:
        import nuvla_forge.kernels as rk
        return rk if rk.HAS_TRITON else None
    except Exception:  # noqa: BLE001 - reference unavailable: skip its column
        return None


def bench_adaln(b, t, n, dtype, peaks, ref):
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda *s: torch.randn(*s, generator=g, device="cuda").to(dtype).requires_grad_(True)  # noqa: E731
    args = {"x": mk(b * t, n), "y": mk(b * t, n), "gate": mk(b, n), "weight": mk(n), "scale": mk(b, n),
            "shift": mk(b, n)}
    dh = torch.randn(b * t, n, device="cuda", dtype=dtype)
    dout = torch.randn(b * t, n, device="cuda", dtype=dtype)

    def run(fn):
        def inner():
            for v in args.values():
                v.grad = None
            h, o = fn(**args, tokens_per_sample=t)
            torch.autograd.backward([h, o], [dh, dout])
        return inner

    res = {"shape": f"B{b}xT{t}xN{n}", "dtype": str(dtype).split(".")[-1]}
    res["eager_ms"] = timeit(run(adaln_residual_rmsnorm_ref))
    from ..ops import norm as _norm
    default = _norm.get_impl()
    for impl, key in ((1, "native_pipelined_ms"), (0, "native_warp_team_ms")):
        _norm.set_impl(impl)
        res[key] = timeit(run(fused_adaln_residual_rmsnorm))
    _norm.set_impl(default)
    res["native_ms"] = res["native_pipelined_ms"] if default == 1 else res["native_warp_team_ms"]
    if ref is not None:
        res["reference_triton_ms"] = timeit(run(ref.fused_adaln_residual_rmsnorm))
    moved = 10 * b * t * n * torch.finfo(dtype).bits // 8
    bw = bandwidth_gb_s(moved, res["native_ms"])
    res.update(bytes=moved, achieved_gb_s=bw, frac_of_measured_hbm=bw / peaks["hbm_gbs"],
               roofline=roofline_note(bw, peaks["hbm_gbs"]), speedup_vs_eager=res["eager_ms"] / res["native_ms"])
    if "reference_triton_ms" in res:
        res["speedup_vs_reference_triton"] = res["reference_triton_ms"] / res["native_ms"]
    return res


def bench_swiglu(m, n, dtype, peaks, ref):
    a = torch.randn(m, n, device="cuda", dtype=dtype, requires_grad=True)
    b = torch.randn(m, n, device="cuda", dtype=dtype, requires_grad=True)
    dout = torch.randn(m, n, device="cuda", dtype=dtype)

    def run(fn):
        def inner():
            a.grad = b.grad = None
            fn(a, b).backward(dout)
        return inner

    res = {"shape": f"{m}x{n}", "dtype": str(dtype).split(".")[-1]}
    res["eager_ms"] = timeit(run(swiglu_ref))
    res["native_ms"] = timeit(run(fused_swiglu))
    if ref is not None:
        res["reference_triton_ms"] = timeit(run(ref.fused_swiglu))
    from .. import _native as nat
    if nat.HAS_NATIVE:
        # the two kernels alone (no autograd between them, L2 flushed before each, device time only)
        out, da, db = (torch.empty(m, n, device="cuda", dtype=dtype) for _ in range(3))
        dc, s = nat.dtype_code(dtype), nat.stream()
        res["native_fwd_kernel_ms"] = timeit_device(lambda: nat.call(
            "nfb_swiglu_fwd", dc, nat.ptr(a), nat.ptr(b), nat.ptr(out), m, n, n, n, n, s))
        res["native_bwd_kernel_ms"] = timeit_device(lambda: nat.call(
            "nfb_swiglu_bwd", dc, nat.ptr(dout), nat.ptr(a), nat.ptr(b), nat.ptr(da), nat.ptr(db), m, n, n, n, n, n, n,
            s))
        kb = bandwidth_gb_s(8 * m * n * torch.finfo(dtype).bits // 8,
                            res["native_fwd_kernel_ms"] + res["native_bwd_kernel_ms"])
        res["kernels_gb_s"], res["kernels_frac_of_measured_hbm"] = kb, kb / peaks["hbm_gbs"]
    moved = 8 * m * n * torch.finfo(dtype).bits // 8
    bw = bandwidth_gb_s(moved, res["native_ms"])
    res.update(bytes=moved, achieved_gb_s=bw, frac_of_measured_hbm=bw / peaks["hbm_gbs"],
               roofline=roofline_note(bw, peaks["hbm_gbs"]), speedup_vs_eager=res["eager_ms"] / res["native_ms"])
    if "reference_triton_ms" in res:
        res["speedup_vs_reference_triton"] = res["reference_triton_ms"] / res["native_ms"]
    return res


def bench_ce(m, h, v, dtype, peaks, ref):
    hid = torch.randn(m, h, device="cuda", dtype=dtype, requires_grad=True)
    w = (torch.randn(v, h, device="cuda") * 0.02).to(dtype).requires_grad_(True)
    tgt = torch.randint(0, v, (m,), device="cuda")
    res = {"shape": f"M{m}xH{h}xV{v}", "dtype": str(dtype).split(".")[-1]}
    cases = [("naive", lambda: chunked_cross_entropy_ref(hid, w, tgt)),
             ("native", lambda: chunked_cross_entropy(hid, w, tgt, chunk_size=1024))]
    if ref is not None:
        cases.append(("reference_triton", lambda: ref.chunked_cross_entropy(hid, w, tgt, chunk_size=1024)))
    for name, fn in cases:
        hid.grad = w.grad = None
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        base = torch.cuda.memory_allocated()
        try:
            ms = timeit(lambda: fn().backward(), iters=5, warmup=2, flush=False)  # noqa: B023
            res[f"{name}_ms"] = ms
            res[f"{name}_peak_mib"] = (torch.cuda.max_memory_allocated() - base) / 2**20
        except torch.OutOfMemoryError:
            res[f"{name}_oom"] = True
    fl = 3 * 2 * m * h * v
    if "native_ms" in res:
        tf = tflops(fl, res["native_ms"])
        res.update(flops=fl, achieved_tflops=tf, frac_of_measured_bf16=tf / peaks["bf16_tflops"],
                   roofline=roofline_note(tf, peaks["bf16_tflops"], "TFLOP/s"))
    if res.get("naive_peak_mib") and res.get("native_peak_mib"):
        res["memory_reduction_vs_naive"] = res["naive_peak_mib"] / res["native_peak_mib"]
    if res.get("reference_triton_ms") and res.get("native_ms"):
        res["speedup_vs_reference_triton"] = res["reference_triton_ms"] / res["native_ms"]
    return res


def bench_patchify(n, hw, p, peaks):
    from ..ops import patchify_images
    from ..ops.image import patch_kpad
    from ..ops.reference import patchify_ref
    img = torch.randint(0, 256, (n, hw, hw, 3), dtype=torch.uint8, device="cuda")
    kpad = patch_kpad(p)
    res = {"shape": f"{n}x{hw}x{hw}x3 p{p}"}
    res["eager_ms"] = timeit(lambda: patchify_ref(img, p, kpad, torch.bfloat16))
    res["native_ms"] = timeit(lambda: patchify_images(img, p))
    moved = img.numel() + n * (hw // p) ** 2 * kpad * 2
    bw = bandwidth_gb_s(moved, res["native_ms"])
    res.update(bytes=moved, achieved_gb_s=bw, frac_of_measured_hbm=bw / peaks["hbm_gbs"],
               roofline=roofline_note(bw, peaks["hbm_gbs"]), speedup_vs_eager=res["eager_ms"] / res["native_ms"])
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="reports/kernels.json")
    ap.add_argument("--quick", action="store_true", help="BASELINE config-2 shapes only")
    ap.add_argument("--no-reference", action="store_true")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("needs a GPU")
    peaks = load_measured_peaks()
    ref = None if args.no_reference else reference_kernels()
    dt = torch.bfloat16
    report = {"device": torch.cuda.get_device_name(0), "peaks": peaks, "reference_triton": ref is not None,
              "adaln": [], "swiglu": [], "cross_entropy": [], "patchify": []}
    adaln_shapes = [(8, 2048, 1536)] + ([] if args.quick else [(8, 32, 384), (8, 128, 384), (16, 256, 768),
                                                                (8, 512, 1024), (4, 1024, 1536)])
    swiglu_shapes = [(16384, 4096)] + ([] if args.quick else [(8192, 1536), (16384, 1536), (32768, 3072)])
    ce_shapes = [(16384, 2048, 32000)] + ([] if args.quick else [(4096, 384, 32000), (16384, 384, 32000)])
    print(f"device {report['device']} | measured peaks: {peaks['hbm_gbs']:.0f} GB/s, "
          f"{peaks['bf16_tflops']:.0f} TFLOP/s ({peaks['source']}) | reference Triton: {ref is not None}")
    for s in adaln_shapes:
        r = bench_adaln(*s, dt, peaks, ref)
        report["adaln"].append(r)
        print(f"adaLN  {r['shape']:<20} eager {r['eager_ms']:7.3f} | ref-triton {r.get('reference_triton_ms', float('nan')):7.3f}"
              f" | native {r['native_ms']:7.3f} ms (pipelined {r['native_pipelined_ms']:.3f}, warp/team "
              f"{r['native_warp_team_ms']:.3f}) | {r['roofline']}")
    for s in swiglu_shapes:
        r = bench_swiglu(*s, dt, peaks, ref)
        report["swiglu"].append(r)
        print(f"SwiGLU {r['shape']:<20} eager {r['eager_ms']:7.3f} | ref-triton {r.get('reference_triton_ms', float('nan')):7.3f}"
              f" | native {r['native_ms']:7.3f} ms | {r['roofline']}")
    for s in ce_shapes:
        r = bench_ce(*s, dt, peaks, ref)
        report["cross_entropy"].append(r)
        print(f"CE     {r['shape']:<20} naive {r.get('naive_ms', float('nan')):7.2f} ms {r.get('naive_peak_mib', 0):7.0f} MiB"
              f" | ref-triton {r.get('reference_triton_ms', float('nan')):7.2f} ms {r.get('reference_triton_peak_mib', 0):7.0f} MiB"
              f" | native {r.get('native_ms', float('nan')):7.2f} ms {r.get('native_peak_mib', 0):7.0f} MiB"
              f" | {r.get('roofline', '')}")
    for s in [(96, 448, 14)]:
        r = bench_patchify(*s, peaks)
        report["patchify"].append(r)
        print(f"patchify {r['shape']:<18} eager {r['eager_ms']:7.3f} | native {r['native_ms']:7.3f} ms | {r['roofline']}")
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(report, indent=2))
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
