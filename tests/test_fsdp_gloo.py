"""FSDP runtime on CPU gloo ranks (world=2): numerics vs single-process AdamW, no_sync, checkpoints."""

import os
import tempfile

import torch
from torch import nn

from _mp import run_ranks


class Block(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.a = nn.Linear(d, 2 * d)
        self.b = nn.Linear(2 * d, d)

    def forward(self, x):
        return x + self.b(torch.tanh(self.a(x)))


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.inp = nn.Linear(12, 16)
        self.blocks = nn.ModuleList([Block(16) for _ in range(3)])
        self.out = nn.Linear(16, 3)
        self.unused = nn.Linear(3, 3)

    def forward(self, x):
        h = self.inp(x)
        for b in self.blocks:
            h = b(h)
        return self.out(h)


def _data(step, rank, m):
    g = torch.Generator().manual_seed(97 * step + 13 * rank + m)
    return torch.randn(6, 12, generator=g), torch.randn(6, 3, generator=g)


def _fsdp_train(rank, world, steps, accum, no_sync, clip):
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    torch.manual_seed(0)
    net = Net()
    fsdp = FullyShardedDataParallel(net, unit_types=(Block,))
    opt = fsdp.make_optimizer(lr=1e-2, weight_decay=0.01, max_grad_norm=clip)
    for step in range(steps):
        for m in range(accum):
            x, y = _data(step, rank, m)
            ctx = fsdp.no_sync() if (no_sync and m < accum - 1) else torch.enable_grad()
            with ctx:
                (((fsdp(x) - y) ** 2).mean() / accum).backward()
        opt.step()
        opt.zero_grad()
    views = fsdp.full_master_views()
    if rank == 0:
        return {n: views[id(p)].clone() for n, p in net.named_parameters()}
    return None


def _reference(world, steps, accum, clip, make=None):
    torch.manual_seed(0)
    net = make() if make is not None else Net()
    opt = torch.optim.AdamW(net.parameters(), lr=1e-2, weight_decay=0.01)
    for step in range(steps):
        opt.zero_grad()
        for r in range(world):
            for m in range(accum):
                x, y = _data(step, r, m)
                (((net(x) - y) ** 2).mean() / (accum * world)).backward()
        for p in net.parameters():
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        if clip > 0:
            torch.nn.utils.clip_grad_norm_(net.parameters(), clip)
        opt.step()
    return {n: p.detach().clone() for n, p in net.named_parameters()}


def _check(out, ref):
    assert all(st == "ok" for st, _ in out.values()), out
    got = out[0][1]
    for n, t in ref.items():
        assert torch.allclose(got[n], t, atol=3e-5), (n, float((got[n] - t).abs().max()))


def test_fsdp_matches_single_process_no_sync_with_global_clip():
    out = run_ranks(_fsdp_train, 2, args=(3, 2, True, 0.5))
    _check(out, _reference(2, 3, 2, 0.5))


def test_fsdp_sync_every_micro_step():
    out = run_ranks(_fsdp_train, 2, args=(2, 2, False, 1.0))
    _check(out, _reference(2, 2, 2, 1.0))


def _fsdp_ckpt(rank, world, path):
    from nuvla_forge_b200.checkpoint import load_checkpoint, save_checkpoint
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    torch.manual_seed(0)
    fsdp = FullyShardedDataParallel(Net(), unit_types=(Block,))
    opt = fsdp.make_optimizer(lr=1e-2)
    x, y = _data(0, rank, 0)
    ((fsdp(x) - y) ** 2).mean().backward()
    opt.step()
    save_checkpoint(path, fsdp, opt, step=1)
    torch.manual_seed(3)
    fsdp2 = FullyShardedDataParallel(Net(), unit_types=(Block,))
    opt2 = fsdp2.make_optimizer(lr=1e-2)
    step = load_checkpoint(path, fsdp2, opt2)
    return {"eq": torch.equal(fsdp.master, fsdp2.master) and torch.equal(opt.m, opt2.m), "step": step}


def test_fsdp_checkpoint_roundtrip():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ck.pt")
        out = run_ranks(_fsdp_ckpt, 2, args=(path,))
        assert all(st == "ok" for st, _ in out.values()), out
        assert out[0][1]["eq"] and out[1][1]["eq"] and out[0][1]["step"] == 1
        sd = torch.load(path, weights_only=False)["model"]
        assert set(sd) == set(Net().state_dict())


def test_unit_layout_puts_1d_params_first():
    """The prefix a fused gather copies ahead holds exactly the unit's 1-D parameters."""
    from nuvla_forge_b200.models import NuVLA, NuVLAConfig
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    model = NuVLA(NuVLAConfig.preset("tiny"))
    f = FullyShardedDataParallel(model, comm="none")
    for u in f.units[:-1]:
        dims = [s.param.dim() for s in u.segs]
        n1 = sum(1 for d in dims if d <= 1)
        assert all(d <= 1 for d in dims[:n1]) and all(d > 1 for d in dims[n1:]), u.name
        end = max((s.start + s.numel + 7) // 8 * 8 for s in u.segs if s.param.dim() <= 1)
        assert u.prefix == end, (u.name, u.prefix, end)
        assert all(s.start >= u.prefix for s in u.segs if s.param.dim() > 1)


def test_rest_copies_cover_unit_minus_prefix_and_weight():
    import random

    from nuvla_forge_b200.parallel.fsdp import rest_copies

    rng = random.Random(0)
    for _ in range(200):
        world = rng.choice([1, 2, 4, 8])
        shard = 16 * rng.randint(1, 5000)
        total = shard * world
        prefix = 16 * rng.randint(0, total // 64)
        wbytes = 16 * rng.randint(1, max(1, (total - prefix) // 32))
        w0 = prefix + 16 * rng.randint(0, (total - prefix - wbytes) // 16)
        for rank in range(world):
            cov = []
            for q, f0, f1 in rest_copies(prefix, (w0, wbytes), total, shard, world, rank):
                assert q * shard <= f0 < f1 <= (q + 1) * shard
                cov.append((f0, f1))
            cov.sort()
            want = [(a, b) for a, b in ((prefix, w0), (w0 + wbytes, total)) if b > a]
            # merge the covered pieces and compare with the wanted ranges
            merged = []
            for a, b in cov:
                if merged and merged[-1][1] == a:
                    merged[-1] = (merged[-1][0], b)
                else:
                    assert not merged or merged[-1][1] < a, "overlap"
                    merged.append((a, b))
            assert merged == want, (merged, want)


def _fsdp_rs_adamw(rank, world, fused):
    """Clipping off, no_sync accumulation: AdamW inside the reduce-scatter (host path) vs the flat step."""
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    torch.manual_seed(0)
    net = Net()
    fsdp = FullyShardedDataParallel(net, comm="gloo", unit_types=(Block,), fuse_rs_adamw=fused)
    opt = fsdp.make_optimizer(lr=1e-2, max_grad_norm=0.0)
    for step in range(3):
        for m in range(2):
            x, y = _data(step, rank, m)
            ctx = fsdp.no_sync() if m == 0 else torch.enable_grad()
            fsdp.final_backward = m == 1
            with ctx:
                (((fsdp(x) - y) ** 2).mean() / 2).backward()
        opt.step()
        opt.zero_grad()
    views = fsdp.full_master_views()
    return ({n: views[id(p)].clone() for n, p in net.named_parameters()} if rank == 0 else None,
            fsdp.fused_steps, opt.step_count)


def test_fsdp_rs_adamw_host_path_matches_flat_step():
    a = run_ranks(_fsdp_rs_adamw, 2, args=(True,))
    b = run_ranks(_fsdp_rs_adamw, 2, args=(False,))
    assert all(st == "ok" for st, _ in a.values()) and all(st == "ok" for st, _ in b.values()), (a, b)
    pa, fused_a, steps_a = a[0][1]
    pb, fused_b, steps_b = b[0][1]
    assert steps_a == steps_b == 3 and fused_a == 3 and fused_b == 0
    for n, t in pb.items():
        assert torch.allclose(pa[n], t, rtol=1e-5, atol=1e-6), n


class _OwnerLinearFn(torch.autograd.Function):
    """The native linear's gradient contract on CPU: dW (fp32) goes to the weight's gradient owner."""

    @staticmethod
    def forward(ctx, x, w, b):
        ctx.save_for_backward(x, w)
        ctx.w_ref = w
        return x @ w.t() + b

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy2, x2 = dy.reshape(-1, dy.shape[-1]), x.reshape(-1, x.shape[-1])
        owner = getattr(ctx.w_ref, "_nfb_grad_owner", None)
        gw = dy2.t().float() @ x2.float()
        if owner is not None:
            buf, overwrite = owner.grad_target(ctx.w_ref)
            buf.view(w.shape).copy_(gw) if overwrite else buf.view(w.shape).add_(gw)
            owner.grad_done(ctx.w_ref)
            gw = None
        return dy @ w, gw, dy2.sum(0)


class OwnerLinear(nn.Linear):
    def forward(self, x):
        return _OwnerLinearFn.apply(x, self.weight, self.bias)


class OwnerBlock(Block):
    def __init__(self, d):
        super().__init__(d)
        self.a, self.b = OwnerLinear(d, 2 * d), OwnerLinear(2 * d, d)


class OwnerNet(Net):
    def __init__(self, twice=False):
        super().__init__()
        self.blocks = nn.ModuleList([OwnerBlock(16) for _ in range(3)])
        self.twice = twice

    def forward(self, x):
        h = self.inp(x)
        for b in self.blocks:
            h = b(b(h)) if self.twice else b(h)
        return self.out(h)


def _fsdp_owner_train(rank, world, steps, accum, twice=False):
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    torch.manual_seed(0)
    net = OwnerNet(twice)
    fsdp = FullyShardedDataParallel(net, unit_types=(Block,))
    assert all(getattr(p, "_nfb_grad_owner", None) is fsdp for p in net.parameters() if p.dim() == 2)
    opt = fsdp.make_optimizer(lr=1e-2, weight_decay=0.01, max_grad_norm=0.5)
    for step in range(steps):
        for m in range(accum):
            x, y = _data(step, rank, m)
            ctx = fsdp.no_sync() if m < accum - 1 else torch.enable_grad()
            with ctx:
                (((fsdp(x) - y) ** 2).mean() / accum).backward()
        opt.step()
        opt.zero_grad()
    views = fsdp.full_master_views()
    if rank == 0:
        return {n: views[id(p)].clone() for n, p in net.named_parameters()}
    return None


def test_fsdp_gradient_owner_protocol_matches_single_process():
    """Weights whose backward writes dW into FSDP's accumulator (as the native linear does) train
    exactly like autograd gradients, with no_sync accumulation and the global clip."""
    out = run_ranks(_fsdp_owner_train, 2, args=(3, 2))
    _check(out, _reference(2, 3, 2, 0.5, make=OwnerNet))


def test_fsdp_gradient_owner_rejects_a_second_gradient():
    out = run_ranks(_fsdp_owner_train, 2, args=(1, 1, True))
    assert all(st != "ok" for st, _ in out.values()), out
    assert all("second gradient" in str(msg) for _, msg in out.values()), out


class CkptBlock(Block):
    """Block recomputed in backward through models.layers.checkpointed, as the model's blocks are."""

    def __init__(self, d):
        super().__init__(d)
        self.grad_checkpoint = True
        self.recomputed = 0

    def forward(self, x):
        from nuvla_forge_b200.models.layers import checkpointed

        return checkpointed(self, self._body, x)

    def _body(self, x):
        if torch.is_grad_enabled() and not torch.is_inference_mode_enabled():
            self.recomputed += 1
        return x + self.b(torch.tanh(self.a(x)))


class CkptNet(Net):
    def __init__(self):
        super().__init__()
        torch.manual_seed(0)  # same parameters as Net() under the same seed
        fresh = Net()
        self.blocks = nn.ModuleList([CkptBlock(16) for _ in range(3)])
        self.load_state_dict(fresh.state_dict())


def _fsdp_ckpt_train(rank, world, steps, accum):
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    torch.manual_seed(0)
    net = CkptNet()
    fsdp = FullyShardedDataParallel(net, unit_types=(CkptBlock,))
    opt = fsdp.make_optimizer(lr=1e-2, weight_decay=0.01, max_grad_norm=0.5)
    for step in range(steps):
        for m in range(accum):
            x, y = _data(step, rank, m)
            ctx = fsdp.no_sync() if m < accum - 1 else torch.enable_grad()
            with ctx:
                (((fsdp(x) - y) ** 2).mean() / accum).backward()
        opt.step()
        opt.zero_grad()
    # each block ran its body twice per micro-step: forward, then the recompute in backward
    assert all(b.recomputed == 2 * steps * accum for b in net.blocks), [b.recomputed for b in net.blocks]
    views = fsdp.full_master_views()
    if rank == 0:
        return {n: views[id(p)].clone() for n, p in net.named_parameters()}
    return None


def test_fsdp_with_activation_checkpointing_matches_single_process():
    """Units recomputed in backward: FSDP's output hook gathers the unit before the recompute reads
    its weights, so training matches the single-process reference."""
    out = run_ranks(_fsdp_ckpt_train, 2, args=(3, 2))
    _check(out, _reference(2, 3, 2, 0.5))


def _fsdp_lazy_flags(rank, world):
    from nuvla_forge_b200.parallel.fsdp import FullyShardedDataParallel

    torch.manual_seed(0)
    net = Net()
    net.blocks[1].grad_checkpoint = True
    fsdp = FullyShardedDataParallel(net, unit_types=(Block,))
    fsdp.fuse_ag_gemm = True      # as on GPUs; record the gather mode instead of gathering lazily
    seen = []
    real = fsdp._gather

    def gather(u, lazy=False):
        seen.append((u.name, lazy))
        return real(u, lazy=False)

    fsdp._gather = gather
    x, y = _data(0, rank, 0)
    with torch.no_grad():
        fsdp(x)
    return seen


def test_fsdp_checkpointed_unit_skips_the_fused_gather():
    """With the GEMM-fused gather on, only a checkpointed unit is gathered in full in forward."""
    out = run_ranks(_fsdp_lazy_flags, 2)
    assert all(st == "ok" for st, _ in out.values()), out
    modes = dict(out[0][1])
    blocks = sorted(n for n in modes if "blocks" in n)
    assert [modes[n] for n in blocks] == [True, False, True], modes
