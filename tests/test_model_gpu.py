"""Model-level checks on the GPU: native path vs reference path, and a Trainer step."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _batch(cfg, b=2, seed=0):
    from nuvla_forge_b200.data import SampleSpec, SyntheticBatchSource

    src = SyntheticBatchSource(SampleSpec.for_model(cfg), b, seed=seed, pin=False)
    return {k: v.cuda() for k, v in src.batch(0).items()}


@pytest.mark.parametrize("preset", ["tiny", "ref"])
def test_native_matches_reference_path(preset):
    from nuvla_forge_b200 import _native as nat
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig

    assert nat.HAS_NATIVE
    over = {"image_size": 64} if preset == "ref" else {}
    cfg_n = NuVLAConfig.preset(preset, **over)
    cfg_r = NuVLAConfig.preset(preset, fused=False, **over)
    torch.manual_seed(0)
    mn = NuVLA(cfg_n).cuda()
    mr = NuVLA(cfg_r).cuda()
    mr.load_state_dict(mn.state_dict())
    b = _batch(cfg_n)
    nat.reset_launch_count()
    torch.manual_seed(1)
    on = mn(b["images"], b["trajectory"], b["text_tokens"], b["text_targets"])
    torch.manual_seed(1)
    orf = mr(b["images"], b["trajectory"], b["text_tokens"], b["text_targets"])
    on["loss"].backward()
    orf["loss"].backward()
    assert nat.launch_count() > 0
    for k in ("plan_loss", "reason_loss", "loss"):
        assert abs(float(on[k]) - float(orf[k])) < 1e-3 * max(1.0, abs(float(orf[k]))), k
    for (name, pn), (_, pr) in zip(mn.named_parameters(), mr.named_parameters()):
        if pr.grad is None:
            continue
        num = float((pn.grad - pr.grad).norm())
        den = float(pr.grad.norm()) + 1e-6
        assert num / den < 2e-2 or num < 1e-5, (name, num / den)


def test_trainer_steps_tiny():
    from nuvla_forge_b200.models import NuVLAConfig
    from nuvla_forge_b200.parallel.dist import setup_distributed
    from nuvla_forge_b200.train import Trainer

    info = setup_distributed()
    cfg = NuVLAConfig.preset("tiny")
    tr = Trainer(cfg, info, grad_accum=2, lr=1e-3)
    losses = []
    batches = [_batch(cfg, 2, seed=s) for s in range(2)]
    for _ in range(6):
        losses.append(float(tr.step(batches)))
    assert all(l == l for l in losses)
    assert losses[-1] < losses[0]
    assert tr.opt.step_count == 6


def test_bf16_model_forward_backward_1b_layer_shapes():
    """One backbone-width transformer block of the 1b config runs through the native path."""
    from nuvla_forge_b200.models.layers import TransformerBlock

    blk = TransformerBlock(2048, 16, kv_heads=8, ffn=5632, causal=True).cuda().to(torch.bfloat16)
    x = torch.randn(2, 3392, 2048, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = blk(x)
    y.float().square().mean().backward()
    assert torch.isfinite(x.grad).all()


def test_graphed_planner_matches_eager():
    """The DiT sampling loop captured in one CUDA graph gives the eager sampler's waypoints."""
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig
    from nuvla_forge_b200.serve import GraphedPlanner

    cfg = NuVLAConfig.preset("tiny")
    torch.manual_seed(0)
    model = NuVLA(cfg).cuda().to(torch.bfloat16).eval()
    for p in model.dit.out.parameters():     # the zero-initialised head would make every plan zero
        torch.nn.init.normal_(p, std=0.1)
    b = _batch(cfg)
    ctx = model.context(b["images"], b["text_tokens"])
    z0 = torch.randn(2, model.dit.horizon, model.dit.traj_dim, device="cuda")
    eager = model.dit.sample(ctx, 4, z0=z0)
    planner = GraphedPlanner(model, batch_size=2, context_len=ctx.shape[1], steps=4)
    assert planner.graph is not None
    got = planner(ctx, z0=z0)
    again = planner(ctx, z0=z0)
    torch.cuda.synchronize()
    assert torch.equal(got, again)
    err = float((got - eager).norm() / (eager.norm() + 1e-6))
    assert err < 2e-2, err
    other = planner(ctx)                     # fresh noise
    assert not torch.equal(other, got)


def test_grad_checkpointing_native_blocks():
    """Every block stack recomputed in backward through the native kernels: more launches, same
    loss, gradients within the tolerance of the reduction order."""
    from nuvla_forge_b200 import _native as nat
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig
    from nuvla_forge_b200.train import set_grad_checkpointing

    cfg = NuVLAConfig.preset("tiny")
    torch.manual_seed(0)
    model = NuVLA(cfg).cuda()
    for blk in model.dit.blocks:
        torch.nn.init.normal_(blk.cond[1].weight, std=0.02)
    b = _batch(cfg)

    def run():
        model.zero_grad(set_to_none=True)
        nat.reset_launch_count()
        torch.manual_seed(1)
        out = model(b["images"], b["trajectory"], b["text_tokens"], b["text_targets"])
        out["loss"].backward()
        torch.cuda.synchronize()
        return float(out["loss"].detach()), nat.launch_count(), {n: p.grad.clone() for n, p in
                                                                  model.named_parameters() if p.grad is not None}

    loss0, n0, g0 = run()
    set_grad_checkpointing(model, "all")
    loss1, n1, g1 = run()
    assert n1 > n0, (n0, n1)
    assert abs(loss1 - loss0) < 1e-4 * max(1.0, abs(loss0))
    assert g0.keys() == g1.keys()
    for name in g0:
        num = float((g1[name] - g0[name]).norm())
        den = float(g0[name].norm()) + 1e-6
        assert num / den < 1e-2 or num < 1e-5, (name, num / den)
