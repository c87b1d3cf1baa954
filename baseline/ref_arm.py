"""Reference arm of bench.py: the UNMODIFIED reference (installed in baseline/_ref) on BASELINE config 3.

The reference's ``NuVLA`` cannot express config 3 (no frames, pooling, separate
backbone width, GQA, causal backbone, 3-wide waypoints). This harness builds
the config-3 architecture from the reference's own public modules and runs
them on the reference's stock training path (its train.py semantics with the
``optimised`` preset: fp32 parameters under bf16 autocast, its Triton kernels,
torch DDP with bucket_cap_mb=100 and gradient_as_bucket_view, no_sync on all
but the last micro-step, clip_grad_norm_(1.0), torch fused AdamW(lr 3e-4,
wd 0.01)). Nothing from nuvla_forge_b200 is imported on this path.

Harness extensions, each the minimum the config needs:
* views x frames are folded into the reference's ``n_views`` (12 images);
* 2x2 average pooling of the ViT tokens and a bias-free projection 1024->2048;
* backbone block = reference RMSNorm + reference SwiGLUMLP(2048, 5632, fused)
  + a GQA (16q/8kv) causal attention written like the reference's Attention
  (fused qkv Linear + F.scaled_dot_product_attention);
* a bias-free 2048->1024 projection of the backbone states, because the
  reference DiT's cross-attention requires a context as wide as the DiT;
* the DiT's in/out projections re-created for 3-wide waypoints.
"""

from __future__ import annotations

import os
import sys
from contextlib import nullcontext

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def _import_reference():
    if not os.path.isdir(os.path.join(REF, "nuvla_forge")):
        return None, "reference not installed in baseline/_ref"
    sys.path.insert(0, REF)
    import nuvla_forge
    if not os.path.abspath(nuvla_forge.__file__).startswith(REF):
        return None, f"nuvla_forge resolved to {nuvla_forge.__file__}, not baseline/_ref"
    return nuvla_forge, None


def build_reference_model(cfg_name: str = "1b"):
    from nuvla_forge.kernels import chunked_cross_entropy
    from nuvla_forge.model.dit import RMSNorm, SwiGLUMLP, TrajectoryDiT
    from nuvla_forge.model.nuvla import MultiViewEncoder, NuVLAConfig

    shapes = {
        "1b": dict(img=448, patch=14, images=12, dv=1024, vdepth=24, vheads=16, pool=2, dt=2048, tdepth=16,
                   theads=16, tkv=8, ffn=5632, dd=1024, ddepth=12, dheads=16, horizon=16, text=320),
        "tiny": dict(img=128, patch=16, images=12, dv=256, vdepth=4, vheads=4, pool=1, dt=256, tdepth=4,
                     theads=4, tkv=4, ffn=704, dd=256, ddepth=4, dheads=4, horizon=8, text=96),
    }[cfg_name]
    s = shapes

    class GQAAttention(nn.Module):
        def __init__(self, dim, heads, kv_heads):
            super().__init__()
            self.h, self.hk, self.dh = heads, kv_heads, dim // heads
            self.qkv = nn.Linear(dim, dim + 2 * kv_heads * self.dh, bias=False)
            self.proj = nn.Linear(dim, dim, bias=False)

        def forward(self, x):
            b, t, c = x.shape
            qkv = self.qkv(x).view(b, t, self.h + 2 * self.hk, self.dh)
            q, k, v = qkv.split([self.h, self.hk, self.hk], dim=2)
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True, enable_gqa=self.hk != self.h)
            return self.proj(o.transpose(1, 2).reshape(b, t, c))

    class BackboneBlock(nn.Module):
        def __init__(self):
            super().__init__()
            self.norm1 = RMSNorm(s["dt"])
            self.attn = GQAAttention(s["dt"], s["theads"], s["tkv"])
            self.norm2 = RMSNorm(s["dt"])
            self.mlp = SwiGLUMLP(s["dt"], s["ffn"], fused=True)

        def forward(self, x):
            x = x + self.attn(self.norm1(x))
            return x + self.mlp(self.norm2(x))

    class RefConfig3(nn.Module):
        def __init__(self):
            super().__init__()
            vcfg = NuVLAConfig(image_size=s["img"], patch_size=s["patch"], n_views=s["images"],
                               vision_dim=s["dv"], vision_depth=s["vdepth"], vision_heads=s["vheads"], fused=True)
            self.encoder = MultiViewEncoder(vcfg)
            self.vision_proj = nn.Linear(s["dv"], s["dt"], bias=False)
            self.text_embed = nn.Embedding(32000, s["dt"])
            self.text_pos = nn.Parameter(torch.randn(1, s["text"], s["dt"]) * 0.02)
            self.blocks = nn.ModuleList([BackboneBlock() for _ in range(s["tdepth"])])
            self.text_norm = RMSNorm(s["dt"])
            self.ctx_proj = nn.Linear(s["dt"], s["dd"], bias=False)
            self.dit = TrajectoryDiT(dim=s["dd"], depth=s["ddepth"], n_heads=s["dheads"], horizon=s["horizon"],
                                     fused=True)
            self.dit.in_proj = nn.Linear(3, s["dd"])
            self.dit.out = nn.Linear(s["dd"], 3)
            nn.init.zeros_(self.dit.out.weight)
            nn.init.zeros_(self.dit.out.bias)
            self.lm_head = nn.Parameter(torch.randn(32000, s["dt"]) * 0.02)

        def forward(self, images, trajectory, text_tokens, text_targets):
            x = self.encoder(images)                         # [B, 12*P, dv]
            b, d = x.shape[0], x.shape[-1]
            if s["pool"] > 1:
                g = s["img"] // s["patch"]
                k = s["pool"]
                x = x.view(b * s["images"], g // k, k, g // k, k, d).mean(dim=(2, 4)).reshape(b, -1, d)
            x = self.vision_proj(x)
            n_img = x.shape[1]
            t = self.text_embed(text_tokens) + self.text_pos
            h = torch.cat([x, t.to(x.dtype)], dim=1)
            for blk in self.blocks:
                h = blk(h)
            h = self.text_norm(h)
            plan = self.dit.flow_loss(trajectory, self.ctx_proj(h))
            th = h[:, n_img:]
            reason = chunked_cross_entropy(th.flatten(0, 1), self.lm_head, text_targets.flatten(), chunk_size=1024)
            return {"loss": plan + reason}

    return RefConfig3(), s


def run_reference(args):
    ref, why = _import_reference()
    if ref is None:
        return {"impl": "reference", "unavailable": why}
    import time

    from nuvla_forge.data.loader import normalise_images
    from nuvla_forge.kernels import HAS_TRITON
    from torch.nn.parallel import DistributedDataParallel as DDP

    sys.path.insert(0, os.path.dirname(HERE))
    from bench import BASELINE_SAMPLES_PER_S, METRIC, ClockSampler, max_ranks, timed_steps, visible_gpu_ids

    if "RANK" in os.environ:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
        rank, world = dist.get_rank(), dist.get_world_size()
    else:
        local, rank, world = 0, 0, 1
        torch.cuda.set_device(0)
    dev = torch.device(f"cuda:{local}")
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    state = {}

    def build(grad_ckpt: bool):
        torch.manual_seed(1234 + rank)
        model, s = build_reference_model(args.model_config)
        if grad_ckpt:
            # the reference's own remedy for activation memory (nuvla_forge/train.py:139-152):
            # recompute the vision encoder blocks in backward
            from torch.utils.checkpoint import checkpoint

            for blk in model.encoder.blocks:
                inner = blk.forward

                def fwd(*a, _inner=inner, **kw):
                    return checkpoint(_inner, *a, use_reentrant=False, **kw)

                blk.forward = fwd
        model = model.to(dev)
        if world > 1:
            model = DDP(model, device_ids=[local], bucket_cap_mb=args.bucket_mb, gradient_as_bucket_view=True)
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.01, fused=True)
        state.update(model=model, opt=opt, s=s, grad_ckpt=grad_ckpt)

    build(False)
    s = state["s"]
    A, B = args.grad_accum, args.batch_size
    gen = torch.Generator().manual_seed(7 + rank)

    def host_batch():
        imgs = torch.randint(0, 256, (B, s["images"], 3, s["img"], s["img"]), dtype=torch.uint8, generator=gen)
        toks = torch.randint(0, 32000, (B, s["text"]), generator=gen)
        tg = torch.full_like(toks, -100)
        n_ins = 64 if args.model_config == "1b" else 32
        tg[:, n_ins - 1: -1] = toks[:, n_ins:]
        traj = torch.randn(B, s["horizon"], 3, generator=gen)
        return {k: v.pin_memory() for k, v in
                {"images": imgs, "trajectory": traj, "text_tokens": toks, "text_targets": tg}.items()}

    def step(micro):
        model, opt = state["model"], state["opt"]
        for m, b in enumerate(micro):
            b = {k: v.to(dev, non_blocking=True) for k, v in b.items()}
            images = normalise_images(b["images"], dtype=torch.bfloat16)
            ctx = model.no_sync() if (world > 1 and m < len(micro) - 1) else nullcontext()
            with ctx, torch.autocast("cuda", dtype=torch.bfloat16):
                out = model(images, b["trajectory"].to(torch.bfloat16), b["text_tokens"], b["text_targets"])
                loss = out["loss"] / len(micro)
            loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return out["loss"].detach()

    n_dev = 2 * A
    dev_batches = [{k: v.to(dev) for k, v in host_batch().items()} for _ in range(n_dev)]
    c = {"i": 0}

    def dev_step():
        i = c["i"]
        c["i"] += 1
        step([dev_batches[(i * A + j) % n_dev] for j in range(A)])

    t0 = time.time()
    try:
        dev_step()
        oom = 0.0
    except torch.OutOfMemoryError:
        oom = 1.0
    # every rank must agree before rebuilding (collective order stays identical)
    if world > 1:
        flag = torch.tensor([oom], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        oom = float(flag.item())
    if oom:
        state.clear()
        import gc

        gc.collect()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
        build(True)
        dev_step()
    for _ in range(max(0, args.warmup - 1)):
        dev_step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(visible_gpu_ids()) if rank == 0 else None
    if sampler:
        sampler.start()
    ms = timed_steps(dev_step, args.steps, dev)
    clocks = sampler.stop() if sampler else None
    ms_step = max_ranks(ms / args.steps, dev)
    gb = B * A * world
    value = gb / (ms_step / 1e3)
    e2e = None
    if not args.no_e2e:
        hb = [[host_batch() for _ in range(A)] for _ in range(args.steps)]
        bytes_in = sum(v.numel() * v.element_size() for b in hb[0] for v in b.values())
        j = {"i": 0}

        def e2e_step():
            loss = step(hb[j["i"]])
            j["i"] += 1
            float(loss.item())

        me = max_ranks(timed_steps(e2e_step, args.steps, dev) / args.steps, dev)
        e2e = {"value": gb / (me / 1e3), "unit": "samples/s", "ms_per_step": me, "h2d_bytes_per_step": int(bytes_in),
               "d2h_bytes_per_step": 4, "api": "reference modules + torch DDP/AdamW (train.py semantics)"}
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "baseline_note": "no published reference number for this config (the reference's 158.05 samples/s is its "
                         "77.3M-param model on 1x H100 NVL)",
        "dtype": "bf16 autocast (fp32 params)",
        "data": "synthetic (uint8 12 images 448px, uniform tokens, random waypoints); random init",
        "config": {"model": f"nuVLA-{args.model_config} from reference modules", "global_batch": gb,
                   "micro_batch_per_gpu": B, "grad_accum": A, "parallelism": f"dp{world}",
                   "bucket_mb": args.bucket_mb, "has_triton": HAS_TRITON,
                   "grad_checkpoint_encoder": state["grad_ckpt"],
                   "l2": "inputs larger than L2"},
        "clocks": clocks, "e2e": e2e, "gpu_launches": None,
        "peak_mem_mib": torch.cuda.max_memory_allocated(dev) / 2**20, "setup_s": time.time() - t0,
    }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return out if rank == 0 else None
