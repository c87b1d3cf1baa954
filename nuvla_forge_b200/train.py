"""Training entry point and the ``Trainer`` API.

    python -m nuvla_forge_b200.train --preset optimised --model-config tiny
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m nuvla_forge_b200.train \
        --preset optimised --model-config 1b --batch-size 8 --grad-accum 4

Parity: nuvla_forge/train.py:41-271 — the same flags and presets
(``--preset {baseline,optimised,custom}``, ``--fused-kernels``, ``--fast-loader``,
``--cuda-prefetch``, ``--bf16``, ``--grad-checkpoint``, ``--ddp-bucket-mb``,
``--no-sync-accum``, ``--fsdp``, ``--compile``, ``--profile``, ...) and the same
``reports/train-<tag>.json`` keys (step_ms, step_ms_mean/p10/p90, n_steps,
<phase>_ms/_pct for data/fwd_bwd/optim, world_size, batch_size, global_batch,
samples_per_sec, peak_mem_mib, flags, model). Added: ``--model-config``
(ref/tiny/1b/3b), ``--comm``, checkpointing (``--save-every``, ``--ckpt-dir``,
``--resume``), ``--max-grad-norm``, ``--native-attention``, ``--no-fused-gather``,
max-over-ranks throughput and exposed
communication in the report. Differences that fix reference bugs: the backend
follows the device (gloo on CPU), each micro-step consumes its own batch,
the gradient norm under FSDP is global, and nothing syncs the host inside a
step except the periodic loss print.

``--bf16`` means bf16 parameters and activations with fp32 master weights
and fp32 gradient accumulation (the reference used fp32 parameters under
autocast); ``--fused-kernels`` selects the native sm_100a kernels (else the
pure-PyTorch references).
"""

from __future__ import annotations

import argparse
import json
import os
from contextlib import nullcontext
from pathlib import Path

import torch

from .checkpoint import load_checkpoint, save_checkpoint
from .data.adapters import SampleSpec, build_dataset
from .data.loader import (CudaPrefetcher, LoaderConfig, SyntheticBatchSource, build_fast_loader,
                          build_naive_loader, describe_environment)
from .health import HealthMonitor
from .models.nuvla import NuVLA, NuVLAConfig
from .optim.adamw import FlatAdamW
from .parallel.ddp import DistributedDataParallel
from .parallel.dist import DistInfo, max_over_ranks, setup_distributed, teardown_distributed
from .profiling import CommTimer, StepTimer, make_profiler, trace

BATCH_KEYS = ("images", "trajectory", "text_tokens", "text_targets")


class Trainer:
    """Model + data-parallel runtime + optimizer; ``step()`` runs one optimizer step.

    This is the public training API (``train.py`` and ``bench.py`` both drive it).
    """

    def __init__(self, cfg: NuVLAConfig, info: DistInfo | None = None, *, lr: float = 3e-4,
                 weight_decay: float = 0.01, max_grad_norm: float = 1.0, bucket_mb: float = 25.0,
                 comm: str = "auto", fsdp: bool = False, grad_accum: int = 1, no_sync_accum: bool = True,
                 bf16: bool = True, grad_checkpoint: bool | str = False, seed: int = 1234, compile: bool = False,
                 fused_gather: bool | None = None, heartbeat_s: float = 0.5, peer_timeout_s: float = 30.0):
        self.info = info or setup_distributed()
        self.cfg = cfg
        self.device = self.info.device
        self.grad_accum = max(1, grad_accum)
        self.no_sync_accum = no_sync_accum
        torch.manual_seed(seed)  # same init on every rank; DDP also broadcasts rank 0's weights
        model = NuVLA(cfg).to(self.device)
        torch.manual_seed(seed + self.info.rank)
        set_grad_checkpointing(model, grad_checkpoint)
        if compile:
            model = torch.compile(model)
        param_dtype = torch.bfloat16 if (bf16 and self.device.type == "cuda") else torch.float32
        if fsdp:
            from .parallel.fsdp import FullyShardedDataParallel
            self.model = FullyShardedDataParallel(model, param_dtype=param_dtype, comm=comm,
                                                  fuse_ag_gemm=fused_gather)
            self.opt = self.model.make_optimizer(lr=lr, weight_decay=weight_decay, max_grad_norm=max_grad_norm)
        else:
            self.model = DistributedDataParallel(model, bucket_cap_mb=bucket_mb, comm=comm, param_dtype=param_dtype)
            self.opt = FlatAdamW(self.model.space, lr=lr, weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                                 ddp=self.model)
        self.module = model
        self.comm_timer = CommTimer() if self.device.type == "cuda" and self.info.world > 1 else None
        if self.comm_timer is not None and hasattr(self.model, "comm_timer"):
            self.model.comm_timer = self.comm_timer
        self.copy_stream = torch.cuda.Stream(self.device) if self.device.type == "cuda" else None
        self.step_count = 0
        hb = None
        if self.info.world > 1 and heartbeat_s > 0:
            from .parallel.watchdog import Heartbeat
            hb = Heartbeat(interval=heartbeat_s).start()
        self.health = HealthMonitor(self.device, self.model, self.info.world, heartbeat=hb, max_age=peer_timeout_s)

    # ------------------------------------------------------------------
    def to_device(self, batch: dict) -> dict:
        """Copy one micro-batch to the device (non-blocking from pinned memory, on the copy stream)."""
        if self.copy_stream is None:
            return {k: batch[k].to(self.device) for k in BATCH_KEYS if k in batch}
        with torch.cuda.stream(self.copy_stream):
            out = {k: batch[k].to(self.device, non_blocking=True) for k in BATCH_KEYS if k in batch}
        return out

    def step(self, micro_batches: list[dict], timer: StepTimer | None = None) -> torch.Tensor:
        """One optimizer step over ``len(micro_batches)`` micro-batches (host or device tensors).

        Host batches are copied on a side stream while earlier micro-steps
        compute. Returns the mean loss as a device tensor (no host sync).
        Before any launch, raises ``PeerLost`` if a peer stopped its heartbeat
        and ``DeviceFault`` if a native kernel's bounded wait gave up during an
        earlier step (read from an asynchronous copy of the status words).
        """
        self.health.before_step()
        n = len(micro_batches)
        on_dev = [self.to_device(b) if not b["images"].is_cuda else b for b in micro_batches] \
            if self.device.type == "cuda" else [{k: b[k] for k in BATCH_KEYS if k in b} for b in micro_batches]
        copied = None
        if self.copy_stream is not None:
            copied = torch.cuda.Event()
            copied.record(self.copy_stream)
            torch.cuda.current_stream(self.device).wait_event(copied)
            cur = torch.cuda.current_stream(self.device)
            for b in on_dev:
                for v in b.values():
                    v.record_stream(cur)
        if timer is not None:
            timer.mark("data")
        total = None
        for m, b in enumerate(on_dev):
            ctx = self.model.no_sync() if (self.no_sync_accum and m < n - 1) else nullcontext()
            if hasattr(self.model, "final_backward"):   # FSDP may fuse AdamW into this backward's reduce-scatters
                self.model.final_backward = m == n - 1
            with ctx:
                with trace(f"forward[{m}]"):
                    out = self.model(b["images"], trajectory=b["trajectory"], text_tokens=b["text_tokens"],
                                     text_targets=b["text_targets"])
                loss = out["loss"]
                with trace(f"backward[{m}]"):
                    (loss / n).backward()
            total = loss.detach() if total is None else total + loss.detach()
        if timer is not None:
            timer.mark("fwd_bwd")
        with trace("optimizer"):
            self.opt.step()
            self.opt.zero_grad(set_to_none=True)
        if timer is not None:
            timer.mark("optim")
        self.step_count += 1
        self.health.after_step()
        return total / n

    def check_health(self) -> None:
        """Synchronous check of every device status word and of the peers' heartbeats."""
        self.health.check_now()
        if hasattr(self.model, "check_health"):
            self.model.check_health()

    def close(self) -> None:
        self.health.close()

    def num_parameters(self) -> int:
        return sum(p.numel() for p in self.module.parameters())


CHECKPOINT_STACKS = ("encoder", "fusion", "text", "dit")


def set_grad_checkpointing(model: NuVLA, parts) -> list[str]:
    """Recompute the blocks of the chosen stacks in backward instead of keeping their activations.

    ``parts``: False / None / "none" (off); True (the vision encoder's blocks, as the reference's
    ``--grad-checkpoint``, nuvla_forge/train.py:139-152); "all"; or stack names from
    ``CHECKPOINT_STACKS`` as a comma-separated string or a sequence. Works on the fused block chain
    the native path runs (``forward_chain``) and on the unfused blocks. Returns the stacks enabled.
    """
    if parts is None or parts is False or parts == "none" or parts == "":
        chosen: list[str] = []
    elif parts is True:
        chosen = ["encoder"]
    elif parts == "all":
        chosen = list(CHECKPOINT_STACKS)
    else:
        chosen = [p.strip() for p in parts.split(",")] if isinstance(parts, str) else list(parts)
    unknown = [p for p in chosen if p not in CHECKPOINT_STACKS]
    if unknown:
        raise ValueError(f"unknown checkpoint stack(s) {unknown}; choose from {CHECKPOINT_STACKS} or 'all'")
    stacks = {"encoder": model.encoder.blocks, "fusion": model.fusion, "text": model.text_blocks,
              "dit": model.dit.blocks}
    for name, blocks in stacks.items():
        for blk in blocks:
            blk.grad_checkpoint = name in chosen
    return chosen


# ----------------------------------------------------------------------
def build_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--preset", choices=["baseline", "optimised", "custom"], default="custom")
    p.add_argument("--model-config", default="ref", choices=["ref", "tiny", "1b", "3b"])
    p.add_argument("--dataset", default="synthetic")
    p.add_argument("--data-root", default=None)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup-steps", type=int, default=20)
    p.add_argument("--batch-size", type=int, default=8)
    p.add_argument("--grad-accum", type=int, default=1)
    p.add_argument("--lr", type=float, default=3e-4)
    p.add_argument("--max-grad-norm", type=float, default=1.0)
    p.add_argument("--num-workers", type=int, default=8)
    p.add_argument("--prefetch-factor", type=int, default=4)
    p.add_argument("--fused-kernels", action="store_true")
    p.add_argument("--fast-loader", action="store_true")
    p.add_argument("--cuda-prefetch", action="store_true")
    p.add_argument("--bf16", action="store_true")
    p.add_argument("--grad-checkpoint", action="store_true",
                   help="recompute the vision encoder's blocks in backward (as the reference)")
    p.add_argument("--grad-checkpoint-blocks", default=None,
                   help="recompute these block stacks in backward: comma-separated from "
                        "encoder,fusion,text,dit, or 'all' (overrides --grad-checkpoint)")
    p.add_argument("--ddp-bucket-mb", type=float, default=25.0)
    p.add_argument("--no-sync-accum", action="store_true")
    p.add_argument("--fsdp", action="store_true")
    p.add_argument("--compile", action="store_true")
    p.add_argument("--comm", default="auto", choices=["auto", "fused", "nccl", "nccl_fp32", "gloo", "none"])
    p.add_argument("--native-attention", action="store_true",
                   help="attention forward on the tcgen05 kernel (backward recomputes through SDPA)")
    p.add_argument("--no-fused-gather", action="store_true",
                   help="FSDP: a separate all-gather before each block instead of the gather-fused GEMM")
    p.add_argument("--synthetic-source", action="store_true",
                   help="feed from the native pinned-batch generator instead of a DataLoader")
    p.add_argument("--profile", action="store_true")
    p.add_argument("--save-every", type=int, default=0)
    p.add_argument("--ckpt-dir", default="checkpoints")
    p.add_argument("--resume", default=None)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--peer-timeout", type=float, default=30.0,
                   help="seconds without a heartbeat after which a peer counts as lost")
    p.add_argument("--inject-failure", action="append", default=[], metavar="RANK:STEP:MODE",
                   help="host-side fault injection for resilience tests: at the start of STEP, rank RANK "
                        "raises (raise), exits without cleanup (exit), stops its heartbeat and hangs (stall), "
                        "or waits N seconds (delayN)")
    p.add_argument("--out", default="reports")
    p.add_argument("--tag", default=None)
    return p.parse_args(argv)


def apply_preset(args):
    if args.preset == "baseline":
        args.fused_kernels = False
        args.fast_loader = False
        args.cuda_prefetch = False
        args.bf16 = False
        args.no_sync_accum = False
        args.ddp_bucket_mb = 25.0
    elif args.preset == "optimised":
        args.fused_kernels = True
        args.fast_loader = True
        args.cuda_prefetch = True
        args.bf16 = True
        args.no_sync_accum = True
        args.ddp_bucket_mb = 100.0
    return args


def _injected(args, rank: int, step: int) -> str | None:
    for spec in args.inject_failure:
        r, s, mode = spec.split(":", 2)
        if int(r) == rank and int(s) == step:
            return mode
    return None


def _inject(mode: str, trainer: "Trainer", rank: int, step: int) -> None:
    """Host-side failure injection between steps (no kernel or collective is in flight)."""
    import time

    if mode == "raise":
        raise RuntimeError(f"injected failure on rank {rank} at step {step}")
    if mode == "exit":
        os._exit(3)
    if mode == "stall":
        if trainer.health.heartbeat is not None:
            trainer.health.heartbeat.stop()
        while True:
            time.sleep(1.0)
    if mode.startswith("delay"):
        time.sleep(float(mode[len("delay"):] or 1.0))
        return
    raise ValueError(f"unknown injection mode {mode!r}")


def make_batches(args, cfg: NuVLAConfig, spec: SampleSpec, info: DistInfo):
    """Micro-batch iterator for the run."""
    if args.synthetic_source and args.dataset == "synthetic":
        return iter(SyntheticBatchSource(spec, args.batch_size, seed=args.seed, rank=info.rank, world=info.world,
                                         copy_stream=None))
    kw = {"spec": spec}
    if args.data_root:
        kw["root"] = args.data_root
    ds = build_dataset(args.dataset, **kw)
    lcfg = LoaderConfig(batch_size=args.batch_size, num_workers=args.num_workers,
                        prefetch_factor=args.prefetch_factor, max_text_len=cfg.max_text_len,
                        vocab_size=cfg.vocab_size)
    sampler = None
    if info.world > 1:
        from torch.utils.data.distributed import DistributedSampler
        sampler = DistributedSampler(ds)
    loader = (build_fast_loader if args.fast_loader else build_naive_loader)(ds, lcfg, sampler=sampler)
    if args.cuda_prefetch and info.device.type == "cuda":
        loader = CudaPrefetcher(loader, info.device)

    def forever():
        epoch = 0
        while True:
            if sampler is not None:
                sampler.set_epoch(epoch)
            yield from loader
            epoch += 1

    return forever()


def main(argv=None):
    args = apply_preset(build_args(argv))
    info = setup_distributed()
    tag = args.tag or args.preset
    cfg = NuVLAConfig.preset(args.model_config, fused=args.fused_kernels)
    spec = SampleSpec.for_model(cfg)
    if args.native_attention:
        from .ops import flash_attn
        flash_attn.enable(True)
    trainer = Trainer(cfg, info, lr=args.lr, max_grad_norm=args.max_grad_norm, bucket_mb=args.ddp_bucket_mb,
                      comm=args.comm, fsdp=args.fsdp, grad_accum=args.grad_accum,
                      no_sync_accum=args.no_sync_accum, bf16=args.bf16,
                      grad_checkpoint=args.grad_checkpoint_blocks or args.grad_checkpoint,
                      seed=args.seed, compile=args.compile, fused_gather=False if args.no_fused_gather else None,
                      peer_timeout_s=args.peer_timeout)
    start_step = 0
    if args.resume:
        start_step = load_checkpoint(args.resume, trainer.model, trainer.opt)
        trainer.opt.step_count = max(trainer.opt.step_count, start_step)
    batches = make_batches(args, cfg, spec, info)
    timer = StepTimer(warmup=args.warmup_steps, device=info.device)
    prof = make_profiler(Path(args.out) / f"trace-{tag}-rank{info.rank}") if args.profile else nullcontext()
    if info.is_main:
        print(f"[{tag}] {trainer.num_parameters() / 1e6:.1f}M params | world={info.world} | device={info.device} "
              f"| comm={getattr(trainer.model, 'comm', 'fsdp')}")
        print(f"[{tag}] env={describe_environment()}")
    total = args.steps + args.warmup_steps
    try:
        _train_loop(args, trainer, batches, timer, prof, info, cfg, start_step, total)
    except BaseException as exc:
        if trainer.health.heartbeat is not None:      # peers learn of it before their next launch
            trainer.health.heartbeat.mark_failed(f"{type(exc).__name__}: {exc}")
        trainer.close()
        raise
    stats = _report(args, trainer, timer, info, cfg, tag)
    trainer.check_health()
    trainer.close()
    if info.world > 1:
        teardown_distributed()
    return stats


def _train_loop(args, trainer, batches, timer, prof, info, cfg, start_step, total):
    with prof as p:
        for step in range(start_step, start_step + total):
            mode = _injected(args, info.rank, step)
            if mode:
                _inject(mode, trainer, info.rank, step)
            timer.start()
            micro = [next(batches) for _ in range(trainer.grad_accum)]
            loss = trainer.step(micro, timer)
            timer.stop()
            if args.profile:
                p.step()
            if step % 25 == 0:
                lv = float(loss.item())
                if info.is_main:
                    print(f"  step {step:5d}  loss {lv:.4f}  {timer.last_ms():.1f} ms")
            if args.save_every and (step + 1) % args.save_every == 0:
                save_checkpoint(Path(args.ckpt_dir) / f"step-{step + 1:07d}.pt", trainer.model, trainer.opt,
                                step + 1, cfg.to_dict())


def _report(args, trainer, timer, info, cfg, tag):
    stats = timer.summary()
    step_ms_max = max_over_ranks(stats["step_ms"], info.device)
    gb = args.batch_size * info.world * trainer.grad_accum
    exposed = trainer.comm_timer.median_ms() if trainer.comm_timer else 0.0
    if trainer.comm_timer:
        trainer.comm_timer.collect()
        exposed = trainer.comm_timer.median_ms()
    stats.update(
        tag=tag, world_size=info.world, batch_size=args.batch_size, global_batch=gb,
        samples_per_sec=gb / (stats["step_ms"] / 1000) if stats["n_steps"] else float("nan"),
        samples_per_sec_max_over_ranks=gb / (step_ms_max / 1000) if stats["n_steps"] else float("nan"),
        exposed_comm_ms=exposed,
        exposed_comm_pct=100.0 * exposed / stats["step_ms"] if stats["n_steps"] else float("nan"),
        peak_mem_mib=torch.cuda.max_memory_allocated(info.device) / 2**20 if info.device.type == "cuda" else 0,
        flags={k: v for k, v in vars(args).items() if isinstance(v, (bool, int, float, str))},
        model=cfg.to_dict(),
    )
    if info.is_main:
        out_dir = Path(args.out)
        out_dir.mkdir(parents=True, exist_ok=True)
        path = out_dir / f"train-{tag}.json"
        path.write_text(json.dumps(stats, indent=2, default=str))
        print(f"\n[{tag}] step {stats['step_ms']:.2f} ms | {stats['samples_per_sec']:.1f} samples/s | "
              f"peak {stats['peak_mem_mib']:.0f} MiB")
        print(f"[{tag}] wrote {path}")
    return stats


if __name__ == "__main__":
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    main()
