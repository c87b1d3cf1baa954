"""Host-side failure detection: per-rank heartbeats through the process group's store.

The reference has no failure detection beyond NCCL defaults and a final
``dist.barrier()`` (nuvla_forge/train.py:265-267). Here each rank runs a
heartbeat thread that stamps ``<prefix>/<rank>`` in the TCP store every
``interval`` seconds, and :meth:`Heartbeat.check_peers` (called by the trainer
between steps, before the next collective is launched) raises ``PeerLost``
when a peer's stamp is older than ``max_age``, or at once when the peer left a
failure notice (:meth:`Heartbeat.mark_failed`, written by a rank whose step
raised, before it exits). Device-side waits in the fused
collectives are bounded separately (csrc/comm.cu) and report through the
symmetric workspace's status word.
"""

from __future__ import annotations

import threading
import time

import torch.distributed as dist


class PeerLost(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store: dist.Store | None = None, rank: int | None = None, world: int | None = None,
                 interval: float = 0.5, prefix: str = "nfb/hb"):
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = store
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval = interval
        self.prefix = prefix
        self._stop = threading.Event()
        self._th: threading.Thread | None = None
        self._failed = False
        self.beat()

    def beat(self) -> None:
        if not self._failed:
            self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def mark_failed(self, reason: str) -> None:
        """Tell the peers this rank is leaving because of ``reason`` (stops the stamps)."""
        self._failed = True
        self._stop.set()
        try:
            self.store.set(f"{self.prefix}/{self.rank}", "failed:" + reason[:200])
        except Exception:  # noqa: BLE001 - store already gone
            pass

    def start(self) -> "Heartbeat":
        def run():
            while not self._stop.wait(self.interval):
                try:
                    self.beat()
                except Exception:  # noqa: BLE001 - store gone: the job is ending
                    return

        self._th = threading.Thread(target=run, daemon=True)
        self._th.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._th is not None:
            self._th.join(timeout=2 * self.interval)

    def _read(self) -> dict[int, str]:
        out = {}
        for r in range(self.world):
            try:
                out[r] = self.store.get(f"{self.prefix}/{r}").decode()
            except Exception:  # noqa: BLE001 - never stamped
                out[r] = "0"
        return out

    def ages(self, raw: dict[int, str] | None = None) -> dict[int, float]:
        now = time.time()
        out = {}
        for r, v in (raw if raw is not None else self._read()).items():
            try:
                out[r] = now - float(v)
            except ValueError:           # a failure notice
                out[r] = float("inf")
        return out

    def check_peers(self, max_age: float = 10.0) -> None:
        raw = self._read()
        failed = {r: v[len("failed:"):] for r, v in raw.items() if r != self.rank and v.startswith("failed:")}
        if failed:
            desc = ", ".join(f"rank {r} failed ({why})" for r, why in sorted(failed.items()))
            raise PeerLost(f"rank {self.rank}: lost peers ({desc})")
        stale = {r: a for r, a in self.ages(raw).items() if r != self.rank and a > max_age}
        if stale:
            desc = ", ".join(f"rank {r} silent {a:.1f}s" for r, a in sorted(stale.items()))
            raise PeerLost(f"rank {self.rank}: lost peers ({desc})")
