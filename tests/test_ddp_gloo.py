"""Multi-process (gloo, world=2) tests of the DDP runtime, optimizer, checkpointing and failure detection."""

import os
import tempfile
import time

import torch
from torch import nn

from _mp import run_ranks


class Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.a = nn.Linear(16, 32)
        self.b = nn.Linear(32, 32)
        self.c = nn.Linear(32, 4)
        self.unused = nn.Linear(4, 4)   # never receives a gradient

    def forward(self, x):
        return self.c(torch.tanh(self.b(torch.tanh(self.a(x)))))


def _data(step, rank, micro):
    g = torch.Generator().manual_seed(1000 * step + 10 * rank + micro)
    return torch.randn(8, 16, generator=g), torch.randn(8, 4, generator=g)


def _ddp_train(rank, world, steps, accum, bucket_mb, record):
    from nuvla_forge_b200.optim import FlatAdamW
    from nuvla_forge_b200.parallel import DistributedDataParallel

    torch.manual_seed(0)
    model = Toy()
    ddp = DistributedDataParallel(model, bucket_cap_mb=bucket_mb)
    order = []
    if record:
        orig = ddp._reduce

        def rec(b, g):
            order.append(b.index)
            return orig(b, g)

        ddp._reduce = rec
    opt = FlatAdamW(ddp.space, lr=1e-2, weight_decay=0.01, max_grad_norm=1.0, ddp=ddp)
    for step in range(steps):
        for m in range(accum):
            x, y = _data(step, rank, m)
            ctx = ddp.no_sync() if m < accum - 1 else torch.enable_grad()
            with ctx:
                loss = ((ddp(x) - y) ** 2).mean() / accum
                loss.backward()
        opt.step()
        opt.zero_grad()
    return {"master": ddp.space.master.clone(), "order": order, "nb": len(ddp.buckets)}


def _single_reference(world, steps, accum):
    torch.manual_seed(0)
    model = Toy()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-2, weight_decay=0.01)
    for step in range(steps):
        opt.zero_grad()
        for r in range(world):
            for m in range(accum):
                x, y = _data(step, r, m)
                (((model(x) - y) ** 2).mean() / (accum * world)).backward()
        for p in model.parameters():
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
    return model


def test_ddp_matches_single_process_with_no_sync_accumulation():
    out = run_ranks(_ddp_train, 2, args=(3, 2, 0.0002, True))
    assert all(st == "ok" for st, _ in out.values()), out
    m0, m1 = out[0][1]["master"], out[1][1]["master"]
    assert torch.equal(m0, m1), "replicas diverged"
    ref = _single_reference(2, 3, 2)
    from nuvla_forge_b200.parallel import FlatParamSpace

    sp = FlatParamSpace(ref, param_dtype=torch.float32, align=16)
    assert torch.allclose(m0, sp.master, atol=2e-5), float((m0 - sp.master).abs().max())
    # tiny buckets: many buckets, launched strictly in index order, once per step
    order = out[0][1]["order"]
    nb = out[0][1]["nb"]
    assert nb > 2
    assert order == list(range(nb)) * 3
    assert out[1][1]["order"] == order


def _ckpt(rank, world, path):
    from nuvla_forge_b200.checkpoint import load_checkpoint, save_checkpoint
    from nuvla_forge_b200.optim import FlatAdamW
    from nuvla_forge_b200.parallel import DistributedDataParallel

    torch.manual_seed(0)
    ddp = DistributedDataParallel(Toy())
    opt = FlatAdamW(ddp.space, lr=1e-2, ddp=ddp)
    x, y = _data(0, rank, 0)
    ((ddp(x) - y) ** 2).mean().backward()
    opt.step()
    save_checkpoint(path, ddp, opt, step=1)
    torch.manual_seed(5)
    ddp2 = DistributedDataParallel(Toy())
    opt2 = FlatAdamW(ddp2.space, lr=1e-2, ddp=ddp2)
    step = load_checkpoint(path, ddp2, opt2)
    return {"eq": torch.equal(ddp.space.master, ddp2.space.master) and torch.equal(opt.m, opt2.m)
            and torch.equal(opt.v, opt2.v), "step": step}


def test_checkpoint_roundtrip_under_ddp():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ck.pt")
        out = run_ranks(_ckpt, 2, args=(path,))
        assert all(st == "ok" for st, _ in out.values()), out
        assert out[0][1]["eq"] and out[1][1]["eq"] and out[0][1]["step"] == 1
        sd = torch.load(path, weights_only=False)["model"]
        assert set(sd) == set(Toy().state_dict()) and all(v.dtype == torch.float32 for v in sd.values())


def _rank_dies(rank, world):
    import torch.distributed as dist

    from nuvla_forge_b200.parallel import DistributedDataParallel

    ddp = DistributedDataParallel(Toy())
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 (host-side)")
    x, y = _data(0, rank, 0)
    t0 = time.time()
    ((ddp(x) - y) ** 2).mean().backward()   # the all-reduce waits for the dead peer
    dist.barrier()
    return time.time() - t0


def test_dead_rank_is_detected_by_timeout():
    t0 = time.time()
    out = run_ranks(_rank_dies, 2, timeout_s=5.0, join_s=90.0)
    assert out[1][0] == "err" and "injected failure" in out[1][1]
    assert out.get(0, ("err", ""))[0] == "err", out.get(0)
    assert time.time() - t0 < 90


def _heartbeat(rank, world):
    from nuvla_forge_b200.parallel.watchdog import Heartbeat, PeerLost

    hb = Heartbeat(interval=0.1)
    if rank == 1:
        return "silent"       # rank 1 stamps once at construction, then never again
    hb.start()
    time.sleep(1.0)
    try:
        hb.check_peers(max_age=0.5)
    except PeerLost as e:
        hb.stop()
        return f"lost: {e}"
    hb.stop()
    return "no detection"


def test_heartbeat_detects_silent_peer():
    out = run_ranks(_heartbeat, 2)
    assert out[0][0] == "ok" and out[0][1].startswith("lost"), out
