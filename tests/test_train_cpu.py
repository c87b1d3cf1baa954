"""BASELINE config 1 plumbing: the tiny nuVLA config trained through the public Trainer / CLI on CPU."""

import json
import os

import torch

from _mp import run_ranks


def _config1(rank, world, ckpt=False):
    from nuvla_forge_b200.data import SampleSpec, SyntheticBatchSource
    from nuvla_forge_b200.models import NuVLAConfig
    from nuvla_forge_b200.parallel.dist import DistInfo
    from nuvla_forge_b200.train import Trainer

    cfg = NuVLAConfig.preset("tiny", fused=False)
    info = DistInfo(rank, world, rank, torch.device("cpu"), "gloo")
    tr = Trainer(cfg, info, grad_accum=2, no_sync_accum=True, bf16=False, seed=0, grad_checkpoint=ckpt)
    src = SyntheticBatchSource(SampleSpec.for_model(cfg), 2, seed=0, rank=rank, world=world, pin=False)
    losses = [float(tr.step([src.batch(2 * s), src.batch(2 * s + 1)])) for s in range(2)]
    return {"losses": losses, "master": tr.model.space.master[:4096].clone(), "params": tr.num_parameters()}


def test_config1_gloo_world2_replicas_agree():
    """Two gloo DDP ranks keep identical replicas; the same run with every block stack recomputed
    in backward (activation checkpointing) trains like the plain one."""
    out = run_ranks(_config1, 2, timeout_s=120, join_s=600)
    assert all(st == "ok" for st, _ in out.values()), out
    a, b = out[0][1], out[1][1]
    assert torch.equal(a["master"], b["master"])
    assert all(l == l and l > 0 for l in a["losses"] + b["losses"])
    assert 20e6 < a["params"] < 40e6
    ckpt = run_ranks(_config1, 2, args=("all",), timeout_s=120, join_s=600)
    assert all(st == "ok" for st, _ in ckpt.values()), ckpt
    for r in (0, 1):
        torch.testing.assert_close(ckpt[r][1]["master"], out[r][1]["master"], rtol=1e-5, atol=1e-6)
        for x, y in zip(ckpt[r][1]["losses"], out[r][1]["losses"]):
            assert abs(x - y) <= 1e-5 * max(1.0, abs(y)), (x, y)


def test_train_cli_writes_report(tmp_path):
    from nuvla_forge_b200.train import main

    stats = main(["--model-config", "tiny", "--steps", "1", "--warmup-steps", "0", "--batch-size", "1",
                  "--num-workers", "0", "--out", str(tmp_path), "--tag", "cpu", "--save-every", "1",
                  "--ckpt-dir", str(tmp_path / "ck"), "--grad-checkpoint-blocks", "fusion,dit"])
    rep = json.loads((tmp_path / "train-cpu.json").read_text())
    for k in ("step_ms", "n_steps", "samples_per_sec", "world_size", "global_batch", "flags", "model",
              "exposed_comm_ms"):
        assert k in rep, k
    assert stats["n_steps"] == 1 and rep["world_size"] == 1
    assert rep["flags"]["grad_checkpoint_blocks"] == "fusion,dit"
    ck = torch.load(tmp_path / "ck" / "step-0000001.pt", weights_only=False)
    assert ck["step"] == 1 and "encoder.patch.weight" in ck["model"]
    assert os.path.getsize(tmp_path / "ck" / "step-0000001.pt") > 1e6


def test_planner_eager_matches_model_plan():
    """GraphedPlanner (eager on CPU) and NuVLA.plan give the same waypoints for the same noise."""
    import torch

    from nuvla_forge_b200.data import SampleSpec, SyntheticBatchSource
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig
    from nuvla_forge_b200.serve import GraphedPlanner

    cfg = NuVLAConfig.preset("tiny", fused=False)
    torch.manual_seed(0)
    model = NuVLA(cfg).eval()
    for p in model.dit.out.parameters():     # the zero-initialised head would make every plan zero
        torch.nn.init.normal_(p, std=0.1)
    b = SyntheticBatchSource(SampleSpec.for_model(cfg), 2, pin=False).batch(0)
    ctx = model.context(b["images"], b["text_tokens"])
    z0 = torch.randn(2, model.dit.horizon, model.dit.traj_dim)
    want = model.plan(b["images"], b["text_tokens"], steps=4, z0=z0)
    planner = GraphedPlanner(model, batch_size=2, context_len=ctx.shape[1], steps=4)
    got = planner(ctx, z0=z0)
    assert got.shape == (2, model.dit.horizon, model.dit.traj_dim)
    assert torch.allclose(got, want, atol=1e-5), float((got - want).abs().max())
    assert float(got.abs().sum()) > 0


def test_trainer_step_emits_named_trace_ranges():
    """forward / backward / optimizer ranges appear in a torch.profiler trace of one step."""
    import torch

    from nuvla_forge_b200.data import SampleSpec, SyntheticBatchSource
    from nuvla_forge_b200.models import NuVLAConfig
    from nuvla_forge_b200.parallel.dist import DistInfo
    from nuvla_forge_b200.train import Trainer

    cfg = NuVLAConfig.preset("tiny", fused=False)
    info = DistInfo(0, 1, 0, torch.device("cpu"), "none")
    tr = Trainer(cfg, info, grad_accum=2, bf16=False)
    src = SyntheticBatchSource(SampleSpec.for_model(cfg), 1, pin=False)
    mbs = [src.batch(0), src.batch(1)]
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        tr.step(mbs)
    names = {e.name for e in prof.events()}
    for want in ("forward[0]", "backward[1]", "optimizer"):
        assert want in names, want
