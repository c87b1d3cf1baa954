"""CPU tests of the data pipeline, profiling helpers, report generator and checkpoint schema."""

import json
import math

import numpy as np
import pytest
import torch


def test_unicycle_trajectory_kinematics():
    from nuvla_forge_b200.data.adapters import SampleSpec, unicycle_trajectory

    spec = SampleSpec(horizon=16, traj_dim=3, speed_range=(0.0, 15.0), yaw_rate_std=0.1, dt=0.5)
    rng = np.random.default_rng(3)
    for _ in range(50):
        t = unicycle_trajectory(spec, rng)
        assert t.shape == (16, 3) and t.dtype == np.float32
        steps = np.diff(np.vstack([np.zeros((1, 2)), t[:, :2]]), axis=0)
        speeds = np.linalg.norm(steps, axis=1) / spec.dt
        assert np.allclose(speeds, speeds[0], atol=1e-4) and 0.0 <= speeds[0] <= 15.0 + 1e-4
        yaw_steps = np.diff(np.concatenate([[0.0], t[:, 2]]))
        assert np.allclose(yaw_steps, yaw_steps[0], atol=1e-6)        # constant yaw rate


def test_synthetic_dataset_records_are_deterministic():
    from nuvla_forge_b200.data import SampleSpec, build_dataset

    spec = SampleSpec(n_views=6, image_size=32, horizon=6, n_frames=2)
    ds = build_dataset("synthetic", spec=spec, n=10)
    a, b = ds[3], ds[3]
    assert a["images"].shape == (12, 32, 32, 3) and a["images"].dtype == np.uint8
    assert np.array_equal(a["images"], b["images"]) and np.array_equal(a["trajectory"], b["trajectory"])
    assert not np.array_equal(ds[4]["images"], a["images"])


def test_hash_tokenizer_and_next_token_targets():
    from nuvla_forge_b200.data.loader import _hash_tokenize, next_token_targets

    ids = _hash_tokenize("Turn left at the light", 8, 32000)
    assert ids.shape == (8,) and (ids[:5] >= 1).all() and (ids[:5] < 32000).all() and (ids[5:] == -100).all()
    assert np.array_equal(ids, _hash_tokenize("turn LEFT at the light", 8, 32000))   # case-folded, stable
    tok, tgt = next_token_targets(np.array([5, 6, 7]), np.array([8, 9]))
    assert tok.tolist() == [5, 6, 7, 8, 9]
    assert tgt.tolist() == [-100, -100, 8, 9, -100]


def test_naive_loader_batches():
    from nuvla_forge_b200.data import LoaderConfig, SampleSpec, build_dataset, build_naive_loader

    spec = SampleSpec(n_views=2, image_size=16, horizon=4)
    ds = build_dataset("synthetic", spec=spec, n=8)
    cfg = LoaderConfig(batch_size=4, num_workers=0, persistent_workers=False, pin_memory=False, max_text_len=12)
    batches = list(build_naive_loader(ds, cfg))
    assert len(batches) == 2
    b = batches[0]
    assert b["images"].shape == (4, 2, 16, 16, 3) and b["images"].dtype == torch.uint8
    assert b["text_tokens"].shape == (4, 12) and b["text_targets"].shape == (4, 12)
    assert (b["text_tokens"] >= 0).all()


def test_profiling_helpers():
    from nuvla_forge_b200.profiling import StepTimer, bandwidth_gb_s, roofline_note

    assert math.isclose(bandwidth_gb_s(2_000_000_000, 1000.0), 2.0)
    assert "roofline" in roofline_note(90.0, 100.0)
    notes = [roofline_note(x, 100.0) for x in (90.0, 60.0, 30.0, 10.0)]
    assert len(set(notes)) == 4
    t = StepTimer(warmup=0, device=torch.device("cpu"))
    for _ in range(3):
        t.start()
        t.mark("data")
        t.mark("fwd_bwd")
        t.stop()
    s = t.summary()
    assert "step_ms" in s


def test_report_generator_never_invents_numbers(tmp_path):
    from nuvla_forge_b200.bench import report

    (tmp_path / "reports").mkdir()
    out = tmp_path / "RESULTS.md"
    report.main(["--reports", str(tmp_path / "reports"), "--out", str(out)])
    text = out.read_text()
    assert text.count("_Not run._") >= 5
    assert not any(ch.isdigit() for ch in text.split("## Training step")[1].split("##")[0])
    (tmp_path / "reports" / "planner.json").write_text(json.dumps(
        {"model": "tiny", "steps": 4, "rows": [{"batch": 1, "eager_ms": 2.0, "graphed_ms": 1.0, "speedup": 2.0}]}))
    report.main(["--reports", str(tmp_path / "reports"), "--out", str(out)])
    assert "| 1 | 2.00 | 1.00 | 2.00x |" in out.read_text()


def test_reference_state_dict_schema():
    """NuVLAConfig() keeps the reference's 180-key fp32 state_dict."""
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig

    with torch.device("meta"):
        m = NuVLA(NuVLAConfig())
    sd = m.state_dict()
    assert len(sd) == 180
    assert tuple(sd["encoder.patch.weight"].shape) == (384, 3, 16, 16)
    for k in ("encoder.blocks.0.mlp.w_gate.weight", "encoder.blocks.0.mlp.w_up.weight",
              "encoder.blocks.0.attn.qkv.weight", "dit.blocks.0.cond.1.weight", "lm_head", "scene_queries",
              "scene_attn.in_proj_weight", "text_embed.weight"):
        assert k in sd, k
    assert all(v.dtype == torch.float32 for v in sd.values())
    assert not any(k.endswith("_zeros") or k.endswith("_ones") for k in sd)
