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
    # kernel microbench: patchify table and the device-only SwiGLU lines come from the JSON
    (tmp_path / "reports" / "kernels.json").write_text(json.dumps({
        "device": "dev", "peaks": {"hbm_gbs": 1000.0, "bf16_tflops": 1.0, "source": "test"},
        "reference_triton": False, "adaln": [], "cross_entropy": [],
        "swiglu": [{"shape": "8x8", "eager_ms": 3.0, "native_ms": 2.0, "achieved_gb_s": 500.0,
                    "frac_of_measured_hbm": 0.5, "native_fwd_kernel_ms": 0.25, "native_bwd_kernel_ms": 0.5,
                    "kernels_gb_s": 900.0, "kernels_frac_of_measured_hbm": 0.9}],
        "patchify": [{"shape": "1x28x28x3 p14", "eager_ms": 1.0, "native_ms": 0.125, "speedup_vs_eager": 8.0,
                      "achieved_gb_s": 600.0, "frac_of_measured_hbm": 0.6}]}))
    report.main(["--reports", str(tmp_path / "reports"), "--out", str(out)])
    text = out.read_text()
    assert "forward 0.250 ms + backward 0.500 ms = 900 GB/s, 90% of measured HBM" in text
    assert "| `1x28x28x3 p14` | 1.000 | 0.125 | 8.00x | 600 | 60% |" in text


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


def test_drivelm_adapter_reads_local_layout(tmp_path):
    """A DriveLM-style tree (QA JSON + camera JPEGs): views resized, missing cameras zero-filled."""
    from PIL import Image

    from nuvla_forge_b200.data import SampleSpec, build_dataset

    cams = ["CAM_FRONT", "CAM_FRONT_RIGHT", "CAM_FRONT_LEFT", "CAM_BACK", "CAM_BACK_LEFT", "CAM_BACK_RIGHT"]
    paths = {}
    for i, cam in enumerate(cams[:5]):          # CAM_BACK_RIGHT missing on disk
        rel = f"nuscenes/samples/{cam}/frame0.jpg"
        (tmp_path / rel).parent.mkdir(parents=True, exist_ok=True)
        Image.new("RGB", (64, 48), color=(40 * i, 100, 200)).save(tmp_path / rel)
        paths[cam] = rel
    paths["CAM_BACK_RIGHT"] = "nuscenes/samples/CAM_BACK_RIGHT/missing.jpg"
    qa = {"scene0": {"key_frames": {"frame0": {"image_paths": paths, "QA": {
        "perception": [{"Q": "What is ahead?", "A": "A car."}],
        "planning": [{"Q": "What should the ego do?", "A": "Slow down."}]}}}}}
    (tmp_path / "v1_0_train_nus.json").write_text(json.dumps(qa))
    spec = SampleSpec(n_views=6, image_size=32, n_frames=2, horizon=4)
    ds = build_dataset("drivelm", root=str(tmp_path), spec=spec)
    assert len(ds) == 2
    rec = ds[1]
    assert rec["images"].shape == (12, 32, 32, 3)
    assert rec["question"] == "What should the ego do?" and rec["answer"] == "Slow down."
    assert rec["images"][0].mean() > 0 and rec["images"][-1].max() == 0   # front present, back-right zeros
    assert rec["trajectory"].shape == (4, 2)


def test_nureasoning_adapter_reads_local_parquet(tmp_path):
    """nuReasoning from a local parquet directory: ego_future becomes the trajectory target."""
    pytest.importorskip("datasets")
    import pyarrow as pa
    import pyarrow.parquet as pq

    from nuvla_forge_b200.data import SampleSpec, build_dataset

    (tmp_path / "data").mkdir()
    table = pa.table({"question": ["Why brake?"], "reasoning": ["Pedestrian crossing."],
                      "ego_future": [[[1.0, 0.0], [2.0, 0.1], [3.0, 0.2]]], "sample_token": ["tok0"]})
    pq.write_table(table, tmp_path / "data" / "train-00000.parquet")
    spec = SampleSpec(n_views=6, image_size=16, horizon=4)
    ds = build_dataset("nureasoning", root=str(tmp_path / "data"), spec=spec)
    rec = ds[0]
    assert rec["answer"] == "Pedestrian crossing." and rec["sample_id"] == "tok0"
    assert rec["images"].shape == (6, 16, 16, 3) and rec["images"].max() == 0        # no camera columns
    np.testing.assert_allclose(rec["trajectory"][:3], [[1.0, 0.0], [2.0, 0.1], [3.0, 0.2]])
    assert (rec["trajectory"][3] == 0).all()


def test_shard_writer_roundtrip(tmp_path):
    """write_shards packs records into tar shards and ShardDataset reads them back."""
    from nuvla_forge_b200.data import SampleSpec, build_dataset
    from nuvla_forge_b200.data import loader as L

    if not hasattr(L, "write_shards") or not hasattr(L, "ShardDataset"):
        pytest.skip("shard writer not exported")
    spec = SampleSpec(n_views=2, image_size=8, horizon=3)
    ds = build_dataset("synthetic", spec=spec, n=5)
    paths = L.write_shards(ds, str(tmp_path), samples_per_shard=2)
    back = L.ShardDataset(paths) if not isinstance(paths, str) else L.ShardDataset(str(tmp_path))
    assert len(back) == 5
    a, b = ds[3], back[3]
    assert np.array_equal(a["images"], b["images"]) and np.allclose(a["trajectory"], b["trajectory"])


def test_hardware_probe_degrades_gracefully(tmp_path):
    """The probe writes every section even without nvidia-smi or a GPU."""
    import subprocess
    import sys

    out = tmp_path / "hw.txt"
    subprocess.run([sys.executable, "-m", "nuvla_forge_b200.utils.probe", "--out", str(out)], check=True,
                   capture_output=True, timeout=120)
    text = out.read_text()
    for section in ("== nvidia-smi", "== topology", "== peer access", "== versions"):
        assert section in text, section
