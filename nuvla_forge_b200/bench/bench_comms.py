"""Collective sweep: fused NVLink collectives vs NCCL.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m nuvla_forge_b200.bench.bench_comms \\
        [--out reports/comms.json] [--max-mb 1024]

Parity: nuvla_forge/bench/bench_comms.py (NCCL all-reduce fp32 vs bf16,
median event-timed latency, ring bus bandwidth 2(N-1)/N * bytes / t). Here,
for bf16 buffers from 1 KB to 1 GB, on every size:

* all-reduce: ``nfb_ar_twoshot`` (fp32 gradient in, bf16 on the wire, fp32
  out, 1/world scale fused) vs NCCL bf16 and NCCL fp32 all_reduce;
* reduce-scatter: ``nfb_rs_push`` (fp32 gradient in with the bf16 cast fused,
  fp32 shard out, scale fused) vs NCCL bf16 reduce_scatter_tensor;
* all-gather: ``nfb_allgather`` (bf16 shards pulled over NVLink) vs NCCL bf16
  all_gather_into_tensor.

Bus bandwidth: all-reduce 2(N-1)/N * bytes / t, reduce-scatter and all-gather
(N-1)/N * bytes / t, bytes = the full bf16 buffer; time = median of the
per-iteration max over ranks. The NVLink reference is 770 GB/s per direction
per GPU (measured peer copy on this pool).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
from pathlib import Path

import torch
import torch.distributed as dist

from .. import _native as nat
from ..parallel.dist import setup_distributed
from ..parallel.symm import SLOT_AG, SLOT_DDP, SLOT_DDP_B, SLOT_RS, SymmetricWorkspace

NVLINK_GBS = 770.0


def _time(fn, iters, warmup, dev):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    out = []
    for _ in range(iters):
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out.append(float(t))
    return statistics.median(out)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="reports/comms.json")
    ap.add_argument("--max-mb", type=float, default=1024.0)
    ap.add_argument("--min-mb", type=float, default=0.0, help="skip sizes below this")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--ctas", type=int, default=0, help="CTAs for the fused kernels (0 = by size)")
    ap.add_argument("--chunk", type=int, default=2048, help="pipelined all-reduce: vectors per slice per step")
    args = ap.parse_args(argv)
    info = setup_distributed()
    rank, world, dev = info.rank, info.world, info.device
    if world < 2:
        raise SystemExit("run under torchrun with 2+ GPUs")
    sizes = []
    b = 1024
    while b <= args.max_mb * 2**20:
        if b >= args.min_mb * 2**20:
            sizes.append(b)
        b *= 4
    maxn = sizes[-1] // 2
    small_cap = 1 << 20   # one-shot all-reduce up to 2 MB of bf16
    ws = SymmetricWorkspace(2 * (maxn * 2 + 256) + 2 * world * small_cap * 2 + 4096, device=dev)
    send, recv = ws.alloc(maxn * 2), ws.alloc(maxn * 2)
    box = ws.alloc(2 * world * small_cap * 2)
    src32 = torch.randn(maxn, device=dev)
    out32 = torch.empty(maxn, device=dev)
    x16 = src32.to(torch.bfloat16)
    shard32 = torch.empty(maxn // world, device=dev)
    full16 = torch.empty(maxn, dtype=torch.bfloat16, device=dev)
    rows = []
    if rank == 0:
        print(f"world={world} device={torch.cuda.get_device_name(dev)} nccl={'.'.join(map(str, torch.cuda.nccl.version()))}")
        print(f"{'bytes':>12} | {'AR fused':>10} {'AR nccl16':>10} {'AR nccl32':>10} | {'RS fused':>10} {'RS nccl':>10} | "
              f"{'AG fused':>10} {'AG nccl':>10}   (bus GB/s)")
    for nbytes in sizes:
        n = nbytes // 2
        n -= n % (8 * world)
        shard = n // world
        # measured on 2 B200s (reports/comms_n2_ctas.json): above 16 MB the fused kernels need ~256
        # CTAs to approach the link rate (all-reduce 145 -> 435 GB/s bus bandwidth from 32 to 256)
        ctas = args.ctas or (16 if nbytes <= 1 << 20 else 64 if nbytes <= 4 << 20 else 132 if nbytes <= 16 << 20 else 256)
        it = args.iters if nbytes < 256 << 20 else max(5, args.iters // 4)
        s = nat.stream(dev)
        # fused all-reduce: fp32 in/out, bf16 wire
        def ar_fused():
            nat.call("nfb_ar_twoshot", ws.bases_ptr(), rank, world, nat.ptr(src32), nat.ptr(out32), n, send, recv,
                     ws.flag_off, SLOT_DDP, 1.0 / world, ws.next_epoch(SLOT_DDP), ws.timeout_ns, nat.ptr(ws.status),
                     ctas, s)
        t16 = x16[:n].clone()
        t32 = src32[:n].clone()
        r = {"bytes": nbytes, "elements": n, "ctas": ctas}
        r["ar_fused_twoshot_ms"] = _time(ar_fused, it, 3, dev)

        def ar_pipe():
            nat.call("nfb_ar_pipelined", ws.bases_ptr(), rank, world, nat.ptr(src32), nat.ptr(out32), n, send, recv,
                     ws.flag_off, SLOT_DDP, SLOT_DDP_B, 1.0 / world, ws.next_epoch(SLOT_DDP), ws.timeout_ns,
                     nat.ptr(ws.status), args.chunk, ctas, s)
        r["ar_fused_pipelined_ms"] = _time(ar_pipe, it, 3, dev)
        if n <= small_cap:
            def ar_one():
                nat.call("nfb_ar_oneshot", ws.bases_ptr(), rank, world, nat.ptr(src32), nat.ptr(out32), n, box,
                         small_cap, ws.flag_off, 5, 1.0 / world, ws.next_epoch(5), ws.timeout_ns, nat.ptr(ws.status),
                         min(ctas, 16), s)
            r["ar_fused_oneshot_ms"] = _time(ar_one, it, 3, dev)
        r["ar_fused_ms"] = min(r["ar_fused_twoshot_ms"], r["ar_fused_pipelined_ms"], r.get("ar_fused_oneshot_ms", 1e9))
        r["ar_nccl_bf16_ms"] = _time(lambda: dist.all_reduce(t16), it, 3, dev)
        r["ar_nccl_fp32_ms"] = _time(lambda: dist.all_reduce(t32), it, 3, dev)
        nat.call("nfb_cast", 0, 1, __import__("ctypes").c_void_p(ws.local_ptr(send)), nat.ptr(src32), n, 1.0, s)

        def rs_fused():   # fp32 gradient in (cast fused), bf16 on the wire, fp32 shard out
            nat.call("nfb_rs_push", ws.bases_ptr(), rank, world, nat.ptr(src32), n, send, ws.flag_off, SLOT_RS,
                     1.0 / world, ws.next_epoch(SLOT_RS), ws.timeout_ns, nat.ptr(ws.status), nat.ptr(shard32), 0,
                     ctas, s)
        rs_out = torch.empty(shard, dtype=torch.bfloat16, device=dev)
        r["rs_fused_ms"] = _time(rs_fused, it, 3, dev)
        r["rs_nccl_ms"] = _time(lambda: dist.reduce_scatter_tensor(rs_out, t16), it, 3, dev)

        def ag_fused():
            nat.call("nfb_allgather", ws.bases_ptr(), rank, world, shard, send, nat.ptr(full16), ws.flag_off, SLOT_AG,
                     ws.next_epoch(SLOT_AG), ws.timeout_ns, nat.ptr(ws.status), ctas, s)
        ag_in = t16[:shard].clone()
        ag_out = torch.empty(n, dtype=torch.bfloat16, device=dev)
        r["ag_fused_ms"] = _time(ag_fused, it, 3, dev)
        r["ag_nccl_ms"] = _time(lambda: dist.all_gather_into_tensor(ag_out, ag_in), it, 3, dev)
        ws.check()
        b16 = n * 2
        ar_f, rs_f = 2 * (world - 1) / world, (world - 1) / world
        for k, f in (("ar_fused", ar_f), ("ar_fused_twoshot", ar_f), ("ar_fused_pipelined", ar_f),
                     ("ar_nccl_bf16", ar_f), ("rs_fused", rs_f), ("rs_nccl", rs_f), ("ag_fused", rs_f),
                     ("ag_nccl", rs_f)):
            r[f"{k}_busbw"] = f * b16 / (r[f"{k}_ms"] * 1e-3) / 1e9
        r["ar_nccl_fp32_busbw"] = ar_f * n * 4 / (r["ar_nccl_fp32_ms"] * 1e-3) / 1e9
        rows.append(r)
        if rank == 0:
            print(f"{nbytes:12d} | {r['ar_fused_busbw']:10.1f} {r['ar_nccl_bf16_busbw']:10.1f} {r['ar_nccl_fp32_busbw']:10.1f} | "
                  f"{r['rs_fused_busbw']:10.1f} {r['rs_nccl_busbw']:10.1f} | {r['ag_fused_busbw']:10.1f} {r['ag_nccl_busbw']:10.1f}"
                  f"   AR twoshot {r['ar_fused_twoshot_busbw']:6.1f} pipelined {r['ar_fused_pipelined_busbw']:6.1f}"
                  f"   fused AR {r['ar_fused_ms']*1e3:8.1f} us vs nccl {r['ar_nccl_bf16_ms']*1e3:8.1f} us")
    if rank == 0:
        rep = {"world_size": world, "device": torch.cuda.get_device_name(dev),
               "nccl_version": ".".join(map(str, torch.cuda.nccl.version())), "nvlink_ref_gbs": NVLINK_GBS,
               "nvls": os.environ.get("NCCL_NVLS_ENABLE", "default"), "rows": rows}
        out = Path(args.out)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps(rep, indent=2))
        print(f"wrote {out}")
    dist.barrier()
    ws.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
