"""Attention forward: the tcgen05 kernel (csrc/attention.cu) vs PyTorch SDPA (cuDNN on B200).

    python -m nuvla_forge_b200.bench.bench_attention [--out reports/attention.json]

Forward and backward are both timed (backward FLOPs = 2.5x the forward's).
Shapes are the attention calls of one BASELINE config-3 micro-batch (8 samples):
the ViT self-attention over 96 images of 1024 patches (16 heads, D 64), the
causal GQA backbone over 3392 tokens (16 q / 8 kv heads, D 128) and the DiT
cross-attention of 16 waypoint queries into the backbone states. FLOPs count
the two GEMMs (4 * B * H * Sq * Sk * D, halved for causal); time = median of
CUDA-event timings with L2 flushed between iterations.
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch
import torch.nn.functional as F

from ..profiling import load_measured_peaks

SHAPES = [  # name, B, Sq, Sk, Hq, Hkv, D, causal
    ("vit self 96x1024 h16 d64", 96, 1024, 1024, 16, 16, 64, False),
    ("backbone causal gqa 8x3392 h16/8 d128", 8, 3392, 3392, 16, 8, 128, True),
    ("dit cross 8x16->3392 h16 d64", 8, 16, 3392, 16, 16, 64, False),
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


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="reports/attention.json")
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    from ..ops import flash_attn

    peaks = load_measured_peaks()
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")
    rows = []
    for name, B, Sq, Sk, Hq, Hkv, D, causal in SHAPES:
        q = torch.randn(B, Sq, Hq, D, device="cuda").to(torch.bfloat16)
        kv = torch.randn(B, Sk, 2 * Hkv, D, device="cuda").to(torch.bfloat16)
        k, v = kv.split([Hkv, Hkv], dim=2)
        native = _time(lambda: flash_attn.attention_fwd(q, k, v, causal), args.iters, flush)
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        sdpa = _time(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=causal, enable_gqa=Hkv != Hq),
                     args.iters, flush)
        flops = 4.0 * B * Hq * Sq * Sk * D * (0.5 if causal else 1.0)
        r = {"shape": name, "native_ms": native, "sdpa_ms": sdpa, "flops": flops,
             "native_tflops": flops / native / 1e9, "sdpa_tflops": flops / sdpa / 1e9,
             "native_frac_of_measured_bf16": flops / native / 1e9 / peaks["bf16_tflops"]}
        # backward: native (pre + main + dQ convert) vs SDPA's backward (autograd of cuDNN SDPA),
        # 2.5x the forward FLOPs (five GEMMs of the forward's size)
        out, lse = flash_attn.attention_fwd(q, k, v, causal)
        dout = torch.randn_like(out)
        nb = _time(lambda: flash_attn.attention_bwd(q, k, v, out, dout, lse, causal), args.iters, flush)
        qr, kr, vr = (t.detach().requires_grad_(True) for t in (qt, kt, vt))
        o_ref = F.scaled_dot_product_attention(qr, kr, vr, is_causal=causal, enable_gqa=Hkv != Hq)
        go = dout.transpose(1, 2)
        sb = _time(lambda: torch.autograd.grad(o_ref, (qr, kr, vr), go, retain_graph=True), args.iters, flush)
        r.update(native_bwd_ms=nb, sdpa_bwd_ms=sb, native_bwd_tflops=2.5 * flops / nb / 1e9,
                 sdpa_bwd_tflops=2.5 * flops / sb / 1e9)
        rows.append(r)
        print(f"{name:<40} fwd native {native:8.3f} ms ({r['native_tflops']:6.0f} TF/s) | SDPA {sdpa:8.3f} ms "
              f"({r['sdpa_tflops']:6.0f} TF/s) || bwd native {nb:8.3f} ms ({r['native_bwd_tflops']:6.0f} TF/s) | "
              f"SDPA {sb:8.3f} ms ({r['sdpa_bwd_tflops']:6.0f} TF/s)", flush=True)
        flash_attn.check_status()
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps({"device": torch.cuda.get_device_name(), "peaks": peaks, "rows": rows}, indent=2))
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
