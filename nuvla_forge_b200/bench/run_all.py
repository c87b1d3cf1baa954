"""Full benchmark sweep: correctness, kernel / GEMM / attention / loader benchmarks, collectives,
the end-to-end A/B and the flagship benchmark at 1..N GPUs, then RESULTS.md.

    python -m nuvla_forge_b200.bench.run_all [--gpus N] [--quick] [--skip-tests]

Parity: scripts/run_all_benchmarks.sh of the reference (hardware probe, tests, kernel
microbenchmarks, dataloader, collectives when more than one GPU is present, baseline vs
optimised training, report). Every stage writes its JSON under reports/; a failing stage is
reported and the sweep goes on, and the exit code is non-zero if any stage failed.
"""

from __future__ import annotations

import argparse
import subprocess
import sys
import time

import torch


def _torchrun(n: int, *args: str) -> list[str]:
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
            "--master-addr", "127.0.0.1", "--master-port", "29533", *args]


def stages(gpus: int, quick: bool, skip_tests: bool) -> list[tuple[str, list[str]]]:
    py = sys.executable
    out = [("hardware", [py, "-m", "nuvla_forge_b200.utils.probe", "--out", "reports/hardware.txt"]),
           ("build", [py, "-m", "nuvla_forge_b200._build"])]
    if not skip_tests:
        out.append(("tests", [py, "-m", "pytest", "tests", "-q", "-x"]))
    out += [
        ("kernels", [py, "-m", "nuvla_forge_b200.bench.bench_kernels", "--out", "reports/kernels.json"]),
        ("gemm", [py, "-m", "nuvla_forge_b200.bench.bench_gemm", "--out", "reports/gemm.json"]
         + (["--quick"] if quick else [])),
        ("attention", [py, "-m", "nuvla_forge_b200.bench.bench_attention", "--out", "reports/attention.json"]),
        ("dataloader", [py, "-m", "nuvla_forge_b200.bench.bench_dataloader", "--out", "reports/dataloader.json"]),
    ]
    if gpus > 1:
        out.append(("comms", _torchrun(gpus, "-m", "nuvla_forge_b200.bench.bench_comms", "--out",
                                       f"reports/comms_n{gpus}.json")))
    steps = "20" if quick else "150"
    for preset in ("baseline", "optimised"):
        cmd = ["-m", "nuvla_forge_b200.train", "--preset", preset, "--steps", steps, "--model-config", "ref"]
        out.append((f"train-{preset}", _torchrun(gpus, *cmd) if gpus > 1 else [py, *cmd]))
    n = 1
    while n <= gpus:
        args = ["bench.py", "--gpus", str(n), "--steps", "4" if quick else "8", "--warmup", "3",
                "--json-out", f"reports/bench_1b_n{n}.json"]
        out.append((f"bench-n{n}", _torchrun(n, *args) if n > 1 else [py, *args]))
        n *= 2
    out.append(("report", [py, "-m", "nuvla_forge_b200.bench.report"]))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=torch.cuda.device_count() if torch.cuda.is_available() else 0)
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--skip-tests", action="store_true")
    ap.add_argument("--dry-run", action="store_true", help="print the stages and exit")
    args = ap.parse_args(argv)
    failed = []
    for name, cmd in stages(max(1, args.gpus), args.quick, args.skip_tests):
        print(f"### {name}: {' '.join(cmd)}", flush=True)
        if args.dry_run:
            continue
        t0 = time.time()
        rc = subprocess.run(cmd).returncode
        print(f"### {name}: exit {rc} in {time.time() - t0:.0f} s", flush=True)
        if rc != 0:
            failed.append(name)
    if failed:
        print(f"failed stages: {', '.join(failed)}")
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main())
