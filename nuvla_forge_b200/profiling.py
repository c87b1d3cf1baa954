"""Step timing, phase breakdown, exposed-communication accounting, profiler and roofline helpers.

Parity: nuvla_forge/profiling.py:25-142 (StepTimer with start/mark/stop/
last_ms/summary, make_profiler, bandwidth_gb_s, roofline_note). Additions:

* ``StepTimer`` works on CPU too (wall clock), so CPU/gloo runs report times
  instead of NaN.
* ``CommTimer`` measures exposed (non-overlapped) communication: the time the
  compute stream spends blocked on the collective stream at the end of
  backward, from events recorded on the compute stream just before and just
  after that wait.
* ``roofline`` helpers take the measured peaks from MEASURED_PEAKS.json-style
  dicts rather than a spec-sheet table.
"""

from __future__ import annotations

import json
import statistics
import time
from pathlib import Path

import torch


class StepTimer:
    """Per-step and per-phase timing (CUDA events on GPUs, wall clock on CPU)."""

    def __init__(self, warmup: int = 20, device=None):
        self.warmup = warmup
        self.device = torch.device(device) if device is not None else None
        self.cuda = torch.cuda.is_available() and (self.device is None or self.device.type == "cuda")
        self.n = 0
        self.steps: list[float] = []
        self.phases: dict[str, list[float]] = {}
        self._events: list = []
        self._last = 0.0

    def _now(self):
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            return e
        return time.perf_counter()

    @staticmethod
    def _ms(a, b) -> float:
        if isinstance(a, float):
            return (b - a) * 1e3
        return a.elapsed_time(b)

    def start(self):
        self.n += 1
        self._events = [("__start__", self._now())]

    def mark(self, name: str):
        self._events.append((name, self._now()))

    def stop(self):
        if not self._events:
            return
        if self.cuda:
            torch.cuda.synchronize(self.device)
        if self.n <= self.warmup:
            return
        t0 = self._events[0][1]
        prev = t0
        for name, e in self._events[1:]:
            self.phases.setdefault(name, []).append(self._ms(prev, e))
            prev = e
        total = self._ms(t0, self._events[-1][1])
        self.steps.append(total)
        self._last = total

    def last_ms(self) -> float:
        return self._last

    def summary(self) -> dict:
        if not self.steps:
            return {"step_ms": float("nan"), "n_steps": 0}
        med = statistics.median(self.steps)
        out = {"step_ms": med, "step_ms_mean": statistics.fmean(self.steps),
               "step_ms_p10": _pct(self.steps, 10), "step_ms_p90": _pct(self.steps, 90),
               "n_steps": len(self.steps)}
        for name, vals in self.phases.items():
            out[f"{name}_ms"] = statistics.median(vals)
            out[f"{name}_pct"] = 100.0 * statistics.median(vals) / med
        return out


def _pct(values, p):
    s = sorted(values)
    k = max(0, min(len(s) - 1, round(p / 100 * (len(s) - 1))))
    return s[k]


def make_profiler(out_dir: str | Path, wait: int = 10, warmup: int = 10, active: int = 10):
    """torch.profiler with a wait/warmup/active schedule writing TensorBoard traces."""
    from torch.profiler import ProfilerActivity, profile, schedule, tensorboard_trace_handler

    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    return profile(activities=acts, schedule=schedule(wait=wait, warmup=warmup, active=active, repeat=1),
                   on_trace_ready=tensorboard_trace_handler(str(out_dir)), record_shapes=True,
                   profile_memory=True, with_stack=False)


def bandwidth_gb_s(bytes_moved: int, ms: float) -> float:
    return bytes_moved / (ms * 1e-3) / 1e9


def tflops(flops: float, ms: float) -> float:
    return flops / (ms * 1e-3) / 1e12


def roofline_note(achieved: float, peak: float, unit: str = "GB/s") -> str:
    """Achieved as a fraction of a peak, with a verdict band (>80, >50, >25 %)."""
    pct = 100.0 * achieved / peak
    if pct > 80:
        verdict = "at the roofline; no headroom left in this kernel"
    elif pct > 50:
        verdict = "healthy; remaining gap is launch overhead and tails"
    elif pct > 25:
        verdict = "underutilised; check occupancy and coalescing"
    else:
        verdict = "poor; likely latency-, launch- or occupancy-bound"
    return f"{achieved:.0f} {unit} = {pct:.0f}% of {peak:.0f} {unit} -- {verdict}"


def load_measured_peaks(path: str | Path | None = None) -> dict:
    """Measured HBM copy GB/s and cuBLAS bf16 TFLOP/s (falls back to the pool's earlier measurement)."""
    p = Path(path) if path else Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                    "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                    "source": "measured"}
        except Exception:  # noqa: BLE001
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


_NVTX = None


def trace(name: str):
    """A named range for traces: a torch.profiler range (shown by ``make_profiler``), plus an NVTX
    range for external tools when ``NFB_NVTX=1``. Costs nothing measurable when no profiler runs."""
    global _NVTX
    if _NVTX is None:
        import os
        _NVTX = os.environ.get("NFB_NVTX", "0") == "1" and torch.cuda.is_available()
    if not _NVTX:
        return torch.profiler.record_function(name)
    return _Both(name)


class _Both:
    def __init__(self, name: str):
        self.name = name
        self.rf = torch.profiler.record_function(name)

    def __enter__(self):
        torch.cuda.nvtx.range_push(self.name)
        self.rf.__enter__()
        return self

    def __exit__(self, *exc):
        self.rf.__exit__(*exc)
        torch.cuda.nvtx.range_pop()
        return False


class CommTimer:
    """Exposed communication: how long the compute stream waited on the collective stream.

    Records an event on the compute stream right before it waits for the
    collective stream at the end of backward, and one right after; the
    difference is the communication that was NOT overlapped with compute.
    """

    def __init__(self):
        self.samples: list[float] = []
        self._pending: list = []

    def bracket(self, before: torch.cuda.Event, after: torch.cuda.Event) -> None:
        self._pending.append((before, after))

    def collect(self) -> None:
        for a, b in self._pending:
            self.samples.append(a.elapsed_time(b))
        self._pending.clear()

    def median_ms(self) -> float:
        return statistics.median(self.samples) if self.samples else 0.0
