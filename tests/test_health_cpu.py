"""Failure detection in the training loop: status words, failure notices and silent peers (CPU, gloo)."""

import time

import pytest
import torch

from _mp import run_ranks


def test_status_word_raises_device_fault():
    """A nonzero status word of any native op is reported with its decoded site."""
    from nuvla_forge_b200.health import DeviceFault, HealthMonitor
    from nuvla_forge_b200.ops import linear

    mon = HealthMonitor(torch.device("cpu"))
    mon.check_now()                                    # nothing set: no error
    fake = torch.tensor([(2 << 24) | 203], dtype=torch.int32)
    linear._status[97] = fake
    try:
        with pytest.raises(DeviceFault, match="gemm@cuda:97: flag timeout at site 203"):
            mon.check_now()
    finally:
        del linear._status[97]


def test_async_status_copy_is_read_before_next_step():
    """The pinned copy queued after a step is checked by the next before_step (here with a fake event)."""
    from nuvla_forge_b200.health import DeviceFault, HealthMonitor

    class Done:
        def query(self):
            return True

    mon = HealthMonitor(torch.device("cpu"))
    mon._host = torch.tensor([0, (1 << 24) | 7], dtype=torch.int32)
    mon._names = ["norm@cuda:0", "collectives"]
    mon._event = Done()
    with pytest.raises(DeviceFault, match="collectives: barrier timeout at site 7"):
        mon.before_step()
    mon.before_step()                                  # the event was consumed: no second report


def _train(rank, world, extra, tmp):
    from nuvla_forge_b200.train import main

    t0 = time.time()
    try:
        main(["--model-config", "tiny", "--steps", "3", "--warmup-steps", "0", "--batch-size", "1",
              "--num-workers", "0", "--out", tmp, "--tag", f"r{rank}", "--synthetic-source",
              "--peer-timeout", "3"] + extra)
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        return {"err": f"{type(exc).__name__}: {exc}", "s": time.time() - t0}
    return {"err": None, "s": time.time() - t0}


def test_failed_rank_is_reported_to_peer_before_its_next_step(tmp_path):
    """Rank 1 raises at the start of step 1; rank 0 learns it from the store before launching step 1."""
    inj = ["--inject-failure", "1:1:raise", "--inject-failure", "0:1:delay1.5"]
    out = run_ranks(_train, 2, args=(inj, str(tmp_path)), timeout_s=20, join_s=240)
    assert out[1][0] == "ok" and "injected failure on rank 1" in out[1][1]["err"], out
    assert out[0][0] == "ok" and out[0][1]["err"].startswith("PeerLost"), out
    assert "rank 1 failed" in out[0][1]["err"]


def test_silent_rank_is_detected_by_heartbeat_age(tmp_path):
    """Rank 1 stops its heartbeat and hangs between steps; rank 0 raises PeerLost (not a hang)."""
    inj = ["--inject-failure", "1:1:stall", "--inject-failure", "0:1:delay4"]
    out = run_ranks(_train, 2, args=(inj, str(tmp_path)), timeout_s=20, join_s=90)   # rank 1 hangs: killed
    assert out.get(0, ("", {}))[0] == "ok", out
    assert out[0][1]["err"].startswith("PeerLost") and "silent" in out[0][1]["err"], out
    assert 1 not in out                                # the stalled rank never reported
