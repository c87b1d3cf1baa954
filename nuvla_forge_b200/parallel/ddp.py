"""Data parallelism: bucketed gradient all-reduce overlapped with backward.

Parity: the reference wraps the model in torch DDP with ``bucket_cap_mb`` and
``gradient_as_bucket_view`` and skips the reduction on ``no_sync`` micro-steps
(nuvla_forge/train.py:157-167, 207-225). This runtime keeps those semantics
and owns the data path:

* Parameters live in a :class:`FlatParamSpace` (bf16 compute copy, fp32
  master, fp32 gradient accumulator). A post-accumulate-grad hook folds each
  bf16 gradient into its fp32 slot (overwrite on the first micro-step, add
  after) and frees it, so gradient accumulation is exact in fp32.
* Buckets are contiguous ranges of the flat space (reverse registration order
  ~ backward order). When the last gradient of a bucket lands on a syncing
  micro-step, the bucket's collective is launched on a side stream while
  backward continues.
* ``comm="fused"`` (default on GPUs): ONE native kernel per bucket does the
  fp32->bf16 cast, the all-reduce over NVLink peer memory and the 1/world
  scale (csrc/comm.cu, nfb_ar_twoshot). ``comm="nccl"``: bf16 NCCL
  all-reduce (the baseline the fused kernel is measured against);
  ``comm="nccl_fp32"``: fp32 NCCL all-reduce as torch DDP does;
  ``comm="gloo"``: CPU process groups (tests).
* ``no_sync()`` suppresses the collective; the gradient stays accumulated.
"""

from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import nn

from .. import _native as nat
from ..profiling import trace
from .flat import FlatParamSpace
from .symm import SLOT_DDP, SLOT_DDP_B, SLOT_DDP_SMALL, SymmetricWorkspace, symmetric_memory_available

ONESHOT_MAX_ELEMS = 256 * 1024   # buckets up to 512 KB of bf16 use the one-barrier all-reduce
AR_CHUNK_VECS = 2048             # pipelined all-reduce: 16 K elements per slice per pipeline step


@dataclass
class Bucket:
    index: int
    start: int
    end: int
    params: list
    pending: int = 0
    ready: bool = False
    launched: bool = False


def _accumulate(dst: torch.Tensor, src: torch.Tensor, overwrite: bool) -> None:
    if dst.is_cuda and nat.HAS_NATIVE and src.is_contiguous() and src.dtype in nat.DT:
        nat.call("nfb_accum", nat.dtype_code(src.dtype), nat.ptr(dst), nat.ptr(src), dst.numel(), 1.0,
                 int(overwrite), nat.stream(dst.device))
    elif overwrite:
        dst.copy_(src)
    else:
        dst.add_(src)


class DistributedDataParallel(nn.Module):
    def __init__(self, module: nn.Module, bucket_cap_mb: float = 25.0, comm: str = "auto",
                 process_group: dist.ProcessGroup | None = None, param_dtype: torch.dtype | None = None,
                 ctas: int = 48, broadcast: bool = True):
        super().__init__()
        self.module = module
        dev = next(module.parameters()).device
        self.device = dev
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        if param_dtype is None:
            param_dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        if comm == "auto":
            if self.world == 1:
                comm = "none"
            elif dev.type == "cuda":
                comm = "fused" if symmetric_memory_available() else "nccl"
            else:
                comm = "gloo"
        self.comm = comm
        self.space = FlatParamSpace(module, param_dtype=param_dtype, device=dev, align=8 * max(self.world, 1))
        if broadcast and self.world > 1:
            with torch.no_grad():
                dist.broadcast(self.space.master, src=0, group=process_group)
            self.space.sync_params_from_master()
        self.buckets = self._make_buckets(bucket_cap_mb)
        self.bucket_of = {}
        for b in self.buckets:
            for p in b.params:
                self.bucket_of[id(p)] = b
        self.require_sync = True
        self._fresh = True            # next backward overwrites the accumulators (after zero_grad)
        self._next_launch = 0         # buckets launch strictly in index order on every rank
        self._seen: set[int] = set()
        self._callback_queued = False
        self.comm_stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self.ctas = ctas
        # "twoshot" (whole-range phases, default: faster on B200) or "pipelined" (chunked phases)
        self.ar_impl = os.environ.get("NFB_AR_IMPL", "twoshot")
        self.ws = None
        if comm == "fused":
            maxb = max(b.end - b.start for b in self.buckets)
            region = (maxb * 2 + 255) // 256 * 256
            self.small_cap = ONESHOT_MAX_ELEMS
            box = 2 * self.world * self.small_cap * 2
            self.ws = SymmetricWorkspace(2 * region + box + 256, group=process_group, device=dev)
            self.send_off = self.ws.alloc(maxb * 2)
            self.recv_off = self.ws.alloc(maxb * 2)
            self.box_off = self.ws.alloc(box)
        # timing of the collective stream (exposed-communication accounting)
        self.comm_events: list[tuple[torch.cuda.Event, torch.cuda.Event]] = []
        self.record_comm_events = False
        self.comm_timer = None   # profiling.CommTimer: brackets the end-of-backward wait
        for s in self.space.segments:
            s.param.register_post_accumulate_grad_hook(self._hook)
            # linear layers on the native GEMM write this parameter's gradient straight into
            # main_grad (grad_target / grad_done below) instead of handing autograd a bf16 tensor
            s.param._nfb_grad_owner = self

    # ------------------------------------------------------------------
    def _make_buckets(self, cap_mb: float) -> list[Bucket]:
        """Cut the flat space at segment boundaries (multiples of 8*world) into ~cap-sized buckets."""
        cap = max(1, int(cap_mb * 2**20 / 4))  # fp32 elements
        buckets: list[Bucket] = []
        cur: list = []
        start = 0
        segs = self.space.segments
        for i, s in enumerate(segs):
            cur.append(s.param)
            seg_end = segs[i + 1].start if i + 1 < len(segs) else self.space.numel
            if seg_end - start >= cap or i + 1 == len(segs):
                buckets.append(Bucket(len(buckets), start, seg_end, cur, pending=len(cur)))
                cur = []
                start = seg_end
        return buckets

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    @contextlib.contextmanager
    def no_sync(self):
        prev = self.require_sync
        self.require_sync = False
        try:
            yield
        finally:
            self.require_sync = prev

    # ------------------------------------------------------------------
    def zero_grad(self) -> None:
        """Start a new accumulation window: the next backward overwrites instead of adding."""
        self._fresh = True

    def _hook(self, p: nn.Parameter) -> None:
        if p.grad is None:
            # autograd still runs this hook when the layer handed its gradient to grad_target /
            # grad_done (it returned None for the weight): nothing left to accumulate
            return
        self._queue_finalize()
        _accumulate(p.main_grad.view(-1), p.grad.view(-1), self._fresh and id(p) not in self._seen)
        p.grad = None
        self._mark_ready(p)

    def _queue_finalize(self) -> None:
        if not self._callback_queued:
            self._callback_queued = True
            torch.autograd.Variable._execution_engine.queue_callback(self._finalize_backward)

    # gradient owner protocol of ops.linear: the GEMM writes the fp32 gradient itself
    def grad_target(self, p: nn.Parameter):
        """(fp32 gradient buffer of ``p``, overwrite?) for a kernel that produces p's whole gradient."""
        self._queue_finalize()
        return p.main_grad, self._fresh and id(p) not in self._seen

    def grad_done(self, p: nn.Parameter) -> None:
        """``p``'s gradient of this backward is complete in its buffer."""
        self._mark_ready(p)

    def _mark_ready(self, p: nn.Parameter) -> None:
        if id(p) in self._seen:
            raise RuntimeError(f"parameter {self.space.segment(p).name} received a second gradient in one "
                               "backward; its bucket may already be reduced")
        self._seen.add(id(p))
        b = self.bucket_of[id(p)]
        b.pending -= 1
        if b.pending == 0:
            b.ready = True
            if self.require_sync and self.comm != "none":
                self._launch_ready()

    def _launch_ready(self) -> None:
        while self._next_launch < len(self.buckets) and self.buckets[self._next_launch].ready:
            self._launch(self.buckets[self._next_launch])
            self._next_launch += 1

    def _launch(self, b: Bucket) -> None:
        with trace(f"ddp.allreduce[{b.start}:{b.end}]"):
            self._launch_impl(b)

    def _launch_impl(self, b: Bucket) -> None:
        b.launched = True
        g = self.space.grads[b.start: b.end]
        if self.comm_stream is None:
            self._reduce(b, g)
            return
        cur = torch.cuda.current_stream(self.device)
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            if self.record_comm_events:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            self._reduce(b, g)
            if self.record_comm_events:
                e1.record()
                self.comm_events.append((e0, e1))

    def _reduce(self, b: Bucket, g: torch.Tensor) -> None:
        scale = 1.0 / self.world
        if self.comm == "fused":
            ws = self.ws
            if g.numel() <= self.small_cap:   # latency-bound: one barrier
                nat.call("nfb_ar_oneshot", ws.bases_ptr(), ws.rank, ws.world, nat.ptr(g), nat.ptr(g), g.numel(),
                         self.box_off, self.small_cap, ws.flag_off, SLOT_DDP_SMALL, scale,
                         ws.next_epoch(SLOT_DDP_SMALL), ws.timeout_ns, nat.ptr(ws.status), 8,
                         nat.stream(self.device))
            elif self.ar_impl == "pipelined":
                nat.call("nfb_ar_pipelined", ws.bases_ptr(), ws.rank, ws.world, nat.ptr(g), nat.ptr(g), g.numel(),
                         self.send_off, self.recv_off, ws.flag_off, SLOT_DDP, SLOT_DDP_B, scale,
                         ws.next_epoch(SLOT_DDP), ws.timeout_ns, nat.ptr(ws.status), AR_CHUNK_VECS, self.ctas,
                         nat.stream(self.device))
            else:
                nat.call("nfb_ar_twoshot", ws.bases_ptr(), ws.rank, ws.world, nat.ptr(g), nat.ptr(g), g.numel(),
                         self.send_off, self.recv_off, ws.flag_off, SLOT_DDP, scale, ws.next_epoch(SLOT_DDP),
                         ws.timeout_ns, nat.ptr(ws.status), self.ctas, nat.stream(self.device))
        elif self.comm == "nccl":
            t = g.to(torch.bfloat16)
            dist.all_reduce(t, group=self.group)
            g.copy_(t.float().mul_(scale))
        else:  # nccl_fp32 / gloo
            dist.all_reduce(g, group=self.group)
            g.mul_(scale)

    def _finalize_backward(self) -> None:
        self._callback_queued = False
        sync = self.require_sync and self.comm != "none"
        if self._fresh:
            # parameters that received no gradient in the first backward of the
            # window still hold the previous window's values: zero them
            for s in self.space.segments:
                if id(s.param) not in self._seen:
                    s.param.main_grad.zero_()
        if sync:
            for b in self.buckets:
                b.ready = True
            self._launch_ready()
            if self.comm_stream is not None:
                cur = torch.cuda.current_stream(self.device)
                if self.comm_timer is not None:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(cur)
                    cur.wait_stream(self.comm_stream)
                    e1.record(cur)
                    self.comm_timer.bracket(e0, e1)
                else:
                    cur.wait_stream(self.comm_stream)
        for b in self.buckets:
            b.pending = len(b.params)
            b.ready = False
            b.launched = False
        self._next_launch = 0
        self._seen.clear()
        self._fresh = False

    # ------------------------------------------------------------------
    def check_health(self) -> None:
        if self.ws is not None:
            self.ws.check()

    @property
    def grad_buffer(self) -> torch.Tensor:
        return self.space.grads

    def state_dict(self, *args, **kwargs):
        return self.module.state_dict(*args, **kwargs)

    def load_state_dict(self, sd, strict: bool = True):
        return self.module.load_state_dict(sd, strict=strict)
