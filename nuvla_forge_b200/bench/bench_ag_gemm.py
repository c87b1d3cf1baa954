"""All-gather fused into the first consuming GEMM (``nfb_ag_gemm``) vs the two-step path.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m nuvla_forge_b200.bench.bench_ag_gemm \\
        [--out reports/ag_gemm_nN.json] [--iters 20]

The cases are the FSDP units of the BASELINE config-4 (3b) model at 4 samples
per GPU, each with the unit's first linear layer: a backbone block (whole
block gathered; qkv GEMM, M = 4 x 3392 tokens), a ViT block (qkv, M = 48
images x 1024 patches) and a DiT block (adaLN conditioning GEMM, M = 4).
For each case, timed with CUDA events (median of the per-iteration max over
ranks, L2 flushed between iterations):

* fused:    ``nfb_ag_gemm`` (gather of the whole unit + the GEMM, one kernel)
* separate: ``nfb_allgather`` of the unit, then the same GEMM by cuBLAS
* separate_ce: the unit gathered by the copy engines (one peer copy per shard), then cuBLAS
* fused_w_ce: ``nfb_ag_gemm`` gathering only W while the copy engines move the rest of the
  unit on a second stream (the FSDP runtime's steady state)
* gemm:     the GEMM alone (cuBLAS, weights already local)

Roofline of the fused kernel = max(GEMM FLOPs / measured bf16 peak, bytes
that cross NVLink / 770 GB/s) with (world-1)/world of the unit crossing
NVLink; ``frac_of_roofline`` = roofline / fused time. With one GPU the gather
is a local copy and only the compute term applies.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import statistics
from pathlib import Path

import torch
import torch.distributed as dist

from .. import _native as nat
from ..parallel.dist import setup_distributed
from ..parallel.symm import SLOT_AG, SymmetricWorkspace
from ..profiling import load_measured_peaks

NVLINK_GBS = 770.0


def _cases():
    from ..models import NuVLA, NuVLAConfig

    cfg = NuVLAConfig.preset("3b")
    with torch.device("meta"):
        m = NuVLA(cfg)
    text_tokens = 12 * 256 + 64 + 256
    out = []
    for name, blk, w, M in (("backbone block -> qkv", m.text_blocks[0], m.text_blocks[0].attn.qkv.weight, 4 * text_tokens),
                            ("vit block -> qkv", m.encoder.blocks[0], m.encoder.blocks[0].attn.qkv.weight, 48 * 1024),
                            ("dit block -> adaLN cond", m.dit.blocks[0], m.dit.blocks[0].cond[1].weight, 4)):
        numel = sum(p.numel() for p in blk.parameters())
        prefix = sum((p.numel() + 7) // 8 * 8 for p in blk.parameters() if p.dim() <= 1)
        out.append({"case": name, "unit_params": numel, "prefix": prefix, "M": M, "N": w.shape[0], "K": w.shape[1]})
    return out


def _timed(fn, iters, dev, flush):
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    ts = []
    for _ in range(iters):
        flush.zero_()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ts.append(float(t))
    return statistics.median(ts)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--orders", default="", help="comma-separated NFB_AG_ORDER values to time the fused kernel "
                                                 "with (gather chunk orders, csrc/ag_gemm.cu); default: the built-in")
    args = ap.parse_args(argv)
    info = setup_distributed()
    rank, world, dev = info.rank, info.world, info.device
    if not dist.is_initialized():
        dist.init_process_group("nccl", rank=0, world_size=1, init_method="tcp://127.0.0.1:29591")
    peaks = load_measured_peaks()
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)
    rows = []
    for c in _cases():
        M, N, K = c["M"], c["N"], c["K"]
        numel = c["unit_params"] + (-c["unit_params"]) % (8 * world)
        shard = numel // world
        ws = SymmetricWorkspace(shard * 2 + 4096, device=dev)
        off = ws.alloc(shard * 2)
        g = torch.Generator(device=dev).manual_seed(rank)
        local = (torch.randn(shard, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        nat.call("nfb_copy_async", ctypes.c_void_p(ws.local_ptr(off)), nat.ptr(local), shard * 2, nat.stream(dev))
        torch.cuda.synchronize(dev)
        dist.barrier()
        full = torch.empty(numel, dtype=torch.bfloat16, device=dev)
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        ready = torch.zeros(1024, dtype=torch.int32, device=dev)
        pre = c["prefix"]
        s = nat.stream(dev)

        def fused():
            nat.call("nfb_ag_gemm", ws.bases_ptr(), rank, world, off, shard * 2, nat.ptr(full), pre * 2, numel * 2,
                     pre * 2, N, K, nat.ptr(x), K, M, nat.ptr(y), N, nat.ptr(ready), nat.ptr(ws.status), s)

        w = full[pre: pre + N * K].view(N, K)

        def allgather():
            nat.call("nfb_allgather", ws.bases_ptr(), rank, world, shard, off, nat.ptr(full), ws.flag_off, SLOT_AG,
                     ws.next_epoch(SLOT_AG), ws.timeout_ns, nat.ptr(ws.status), 32, s)

        def separate():
            allgather()
            torch.matmul(x, w.t(), out=y)

        def gemm():
            torch.matmul(x, w.t(), out=y)

        side = torch.cuda.Stream(device=dev)

        def fused_w_ce():
            # the fused kernel gathers only W; the copy engines move the rest of the unit meanwhile
            side.wait_stream(torch.cuda.current_stream(dev))
            hs = ctypes.c_void_p(side.cuda_stream)
            w_lo, w_hi = pre * 2, pre * 2 + N * K * 2
            for i in range(world):
                q = (rank + 1 + i) % world
                for lo, hi in ((0, w_lo), (w_hi, numel * 2)):
                    f0, f1 = max(lo, q * shard * 2), min(hi, (q + 1) * shard * 2)
                    if f1 > f0:
                        nat.call("nfb_copy_async", ctypes.c_void_p(full.data_ptr() + f0),
                                 ctypes.c_void_p(ws.bases[q] + off + (f0 - q * shard * 2)), f1 - f0, hs)
            nat.call("nfb_ag_gemm", ws.bases_ptr(), rank, world, off, shard * 2, nat.ptr(full), w_lo, w_hi,
                     pre * 2, N, K, nat.ptr(x), K, M, nat.ptr(y), N, nat.ptr(ready), nat.ptr(ws.status), s)
            torch.cuda.current_stream(dev).wait_stream(side)

        def separate_ce():
            for i in range(world):
                q = (rank + i) % world
                nat.call("nfb_copy_async", ctypes.c_void_p(full.data_ptr() + q * shard * 2),
                         ctypes.c_void_p(ws.bases[q] + off), shard * 2, s)
            torch.matmul(x, w.t(), out=y)

        r = dict(c, world=world)
        import os
        for o in [x for x in args.orders.split(",") if x]:
            os.environ["NFB_AG_ORDER"] = o
            r[f"fused_order{o}_ms"] = _timed(fused, args.iters, dev, flush)
            if rank == 0:
                print(f"  {c['case']:<26} order {o}: fused {r[f'fused_order{o}_ms']:.3f} ms")
        os.environ.pop("NFB_AG_ORDER", None)
        r["fused_ms"] = _timed(fused, args.iters, dev, flush)
        ws.check()
        r["separate_ms"] = _timed(separate, args.iters, dev, flush)
        r["separate_ce_ms"] = _timed(separate_ce, args.iters, dev, flush)
        r["fused_w_ce_ms"] = _timed(fused_w_ce, args.iters, dev, flush)
        ws.check()
        r["gemm_ms"] = _timed(gemm, args.iters, dev, flush)
        r["allgather_ms"] = _timed(allgather, args.iters, dev, flush)
        ws.check()
        flops = 2.0 * M * N * K
        link_bytes = numel * 2 * (world - 1) / world
        t_compute = flops / (peaks["bf16_tflops"] * 1e12) * 1e3
        t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
        r.update(flops=flops, nvlink_bytes=link_bytes, roofline_ms=max(t_compute, t_link),
                 roofline_bound="compute" if t_compute >= t_link else "nvlink")
        r["frac_of_roofline"] = r["roofline_ms"] / r["fused_ms"]
        r["speedup_vs_separate"] = r["separate_ms"] / r["fused_ms"]
        rows.append(r)
        if rank == 0:
            print(f"{c['case']:<26} M{M} N{N} K{K} unit {numel * 2 / 2**20:7.1f} MiB | fused {r['fused_ms']:.3f} ms"
                  f" | separate {r['separate_ms']:.3f} (AG {r['allgather_ms']:.3f} + GEMM {r['gemm_ms']:.3f})"
                  f" | copy-engine AG + GEMM {r['separate_ce_ms']:.3f} | fused W + copy-engine rest "
                  f"{r['fused_w_ce_ms']:.3f}"
                  f" | roofline {r['roofline_ms']:.3f} ({r['roofline_bound']}) = {100 * r['frac_of_roofline']:.0f}%")
        dist.barrier()
        ws.close()
        del full, x, y
    if rank == 0:
        out = Path(args.out or f"reports/ag_gemm_n{world}.json")
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps({"world_size": world, "device": torch.cuda.get_device_name(dev),
                                   "peaks": peaks, "nvlink_ref_gbs": NVLINK_GBS, "rows": rows}, indent=2))
        print(f"wrote {out}")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
