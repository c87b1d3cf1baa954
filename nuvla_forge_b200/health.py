"""Failure detection between training steps, without synchronising the host.

The reference has no failure detection beyond NCCL defaults and a final
``dist.barrier()`` (nuvla_forge/train.py:265-267). Here two sources are
watched by :class:`HealthMonitor`, which the trainer calls around every step:

* device status words: every bounded wait in the native kernels (tcgen05 GEMM
  and cross-entropy pipelines, norm copy rings, attention, the fused NVLink
  collectives) writes an error code into a device word instead of hanging.
  After each step the monitor copies all words into one pinned host buffer
  (asynchronous device-to-host copies on the compute stream, then an event);
  before the next step it reads the buffer if the event has completed, so a
  failed wait is reported one step later at the latest, and no ``.item()``
  stalls the host;
* peers: with more than one rank, a :class:`parallel.watchdog.Heartbeat`
  thread stamps this rank in the process group's store and ``before_step``
  raises ``PeerLost`` when a peer's stamp is older than ``max_age`` seconds,
  before this rank launches the step's first collective.
"""

from __future__ import annotations

import torch

from .parallel.symm import decode_status


class DeviceFault(RuntimeError):
    """A native kernel's bounded wait gave up (the status word says where)."""


def status_words(model=None) -> list[tuple[str, torch.Tensor]]:
    """Every device status word the native ops and the parallel runtime have created so far."""
    from .ops import ce_tc, flash_attn, linear, norm

    out = []
    for name, mod in (("gemm", linear), ("cross_entropy", ce_tc), ("norm", norm), ("attention", flash_attn)):
        for idx, t in sorted(getattr(mod, "_status", {}).items()):
            out.append((f"{name}@cuda:{idx}", t))
    ws = getattr(model, "ws", None)
    if ws is not None and getattr(ws, "status", None) is not None:
        out.append(("collectives", ws.status))
    return out


class HealthMonitor:
    def __init__(self, device: torch.device, model=None, world: int = 1, heartbeat=None, max_age: float = 30.0):
        self.device = device
        self.model = model
        self.world = world
        self.heartbeat = heartbeat
        self.max_age = max_age
        self._host: torch.Tensor | None = None
        self._names: list[str] = []
        self._event: torch.cuda.Event | None = None
        self.checks = 0

    # ------------------------------------------------------------------
    def after_step(self) -> None:
        """Queue the copies of all status words to pinned host memory (no wait)."""
        if self.device.type != "cuda":
            return
        words = [(n, t) for n, t in status_words(self.model) if t.device == self.device]
        if not words:
            return
        if self._host is None or self._host.numel() < len(words):
            self._host = torch.zeros(max(8, 2 * len(words)), dtype=torch.int32, pin_memory=True)
        for i, (_, t) in enumerate(words):
            self._host[i: i + 1].copy_(t.view(-1)[:1], non_blocking=True)
        self._names = [n for n, _ in words]
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._event = ev

    def before_step(self) -> None:
        """Raise if a peer went silent or a completed status copy shows a failed wait."""
        if self.heartbeat is not None:
            self.heartbeat.check_peers(self.max_age)
        ev = self._event
        if ev is not None and ev.query():
            self._event = None
            self._raise_if_bad()

    def check_now(self) -> None:
        """Synchronous check of every status word (used outside the step loop)."""
        if self.heartbeat is not None:
            self.heartbeat.check_peers(self.max_age)
        for name, t in status_words(self.model):
            v = int(t.view(-1)[0].item())
            if v:
                raise DeviceFault(f"{name}: {decode_status(v & 0xFFFFFFFF)}")

    def _raise_if_bad(self) -> None:
        self.checks += 1
        vals = self._host[: len(self._names)].tolist()
        bad = [(n, v) for n, v in zip(self._names, vals) if v]
        if bad:
            desc = "; ".join(f"{n}: {decode_status(v & 0xFFFFFFFF)}" for n, v in bad)
            raise DeviceFault(f"native kernel wait gave up ({desc})")

    def close(self) -> None:
        if self.heartbeat is not None:
            self.heartbeat.stop()
            self.heartbeat = None
