"""Throughput of back-to-back tcgen05.mma by shape and operand source, on every SM.

    python -m nuvla_forge_b200.bench.bench_mma_rates [--out reports/mma_rates.json]

Each SM runs one CTA whose single thread issues `iters` M128 x N x K16 bf16 MMAs back to back into
one TMEM accumulator (``nfb_mma_rate``); reported: SM cycles per instruction and FLOP per cycle per
SM against the nominal 8192 (2.25 PFLOP/s dense bf16 over 148 SMs at 1.86 GHz). The attention
kernels are built from N = 64 / 128 instructions with A from shared memory or TMEM, so their MMA
time is set by these rates, not by the large-N GEMM rate.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

CASES = [  # mode, n, description
    (0, 256, "A, B shared memory (K-major), N 256"),
    (0, 128, "A, B shared memory (K-major), N 128"),
    (0, 64, "A, B shared memory (K-major), N 64"),
    (1, 128, "B MN-major, N 128"),
    (1, 64, "B MN-major, N 64"),
    (2, 128, "A from TMEM, B MN-major, N 128"),
    (2, 64, "A from TMEM, B MN-major, N 64"),
]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=4096)
    ap.add_argument("--out", default="reports/mma_rates.json")
    args = ap.parse_args(argv)
    from .. import _native as nat

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    rows = []
    for mode, n, desc in CASES:
        nat.call("nfb_mma_rate", mode, n, args.iters, nat.ptr(out), sms, nat.stream())
        torch.cuda.synchronize()
        cycles, ok = (int(v) for v in out.tolist())
        per = cycles / args.iters
        flop = 2.0 * 128 * n * 16
        rows.append({"mode": mode, "n": n, "operands": desc, "cycles_per_instr": per, "flop_per_clk_per_sm": flop / per,
                     "frac_of_8192": flop / per / 8192.0, "completed": bool(ok)})
        print(f"M128 N{n:<3} K16  {desc:<40} {per:6.1f} cycles/instr  {flop / per:6.0f} FLOP/clk/SM "
              f"({100 * flop / per / 8192:.0f}% of 8192)", flush=True)
    Path(args.out).parent.mkdir(parents=True, exist_ok=True)
    Path(args.out).write_text(json.dumps({"device": torch.cuda.get_device_name(), "sms": sms, "iters": args.iters,
                                          "rows": rows}, indent=2))
    print(f"wrote {args.out}")


if __name__ == "__main__":
    main()
