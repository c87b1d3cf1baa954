"""Hardware / software probe written to reports/hardware.txt.

    python -m nuvla_forge_b200.utils.probe [--out reports/hardware.txt]

Parity: scripts/probe_hardware.sh of the reference (nvidia-smi, topology,
peer-access matrix, versions). Read-only: it changes no GPU setting.
"""

from __future__ import annotations

import argparse
import subprocess
from pathlib import Path

import torch


def _run(cmd: list[str]) -> str:
    try:
        return subprocess.run(cmd, capture_output=True, text=True, timeout=60).stdout.strip()
    except Exception as exc:  # noqa: BLE001 - tool missing: record it
        return f"({' '.join(cmd)} unavailable: {exc})"


def probe() -> str:
    out = ["== nvidia-smi", _run(["nvidia-smi", "--query-gpu=index,name,memory.total,clocks.max.sm,power.limit",
                                  "--format=csv"]), "", "== topology", _run(["nvidia-smi", "topo", "-m"]), ""]
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    out.append(f"== peer access ({n} devices)")
    for i in range(n):
        out.append(" ".join("x" if i == j else ("1" if torch.cuda.can_device_access_peer(i, j) else "0")
                            for j in range(n)))
    out += ["", "== versions", f"torch {torch.__version__} cuda {torch.version.cuda}",
            f"nccl {'.'.join(map(str, torch.cuda.nccl.version())) if n else 'n/a'}",
            _run(["nvcc", "--version"]).splitlines()[-1] if _run(["nvcc", "--version"]) else "nvcc n/a"]
    try:
        from .. import _native as nat
        out.append(f"native library: {nat.lib_path()} loaded={nat.HAS_NATIVE}")
    except Exception as exc:  # noqa: BLE001
        out.append(f"native library: {exc}")
    return "\n".join(out) + "\n"


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="reports/hardware.txt")
    args = ap.parse_args(argv)
    text = probe()
    Path(args.out).parent.mkdir(parents=True, exist_ok=True)
    Path(args.out).write_text(text)
    print(text)


if __name__ == "__main__":
    main()
