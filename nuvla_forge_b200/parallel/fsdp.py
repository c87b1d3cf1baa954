"""Fully sharded data parallelism (ZeRO-3) with fused NVLink collectives.

Parity: the reference wraps the whole model in torch FSDP with no wrap policy
(one flat parameter, fp32 parameters, per-rank gradient-norm clipping,
nuvla_forge/train.py:158-160, 228). This runtime shards per block and fixes the
clipping:

* Units: every ``TransformerBlock`` and ``DiTBlock`` is a unit; all remaining
  parameters form the root unit. A unit's parameters are flattened (padded to
  a multiple of 8*world) and split into ``world`` contiguous shards.
* Each rank keeps, for its shard of every unit, an fp32 master copy, AdamW
  moments and an fp32 gradient in ONE flat shard space (so the optimizer is one
  launch), and the bf16 parameter shard in peer-mapped memory, where the
  optimizer writes it directly.
* Forward: before a unit runs, its bf16 parameters are all-gathered into a
  full buffer the module's parameters are views of; after it runs, the
  buffer's storage is released (``reshard_after_forward``). For transformer
  and DiT blocks (``fuse_ag_gemm``) the gather is fused into the block's first
  linear layer: the 1-D parameters (norm weights, biases; laid out first in
  the unit) are copied ahead by the copy engine, and the block's first GEMM is
  ``nfb_ag_gemm`` -- one kernel that pulls the weight it consumes over NVLink
  while its tensor-core tiles consume the weight's row blocks as they land.
  With more than two ranks (``ag_hybrid``), once the consuming weight is known
  (after a unit's first forward) the kernel gathers only that weight and the
  rest of the unit goes to the copy engines on the prefetch stream,
  concurrently. The root unit's gather opens every step with the
  ``nfb_allgather`` kernel, whose rank barrier is what makes every later
  gather of the step safe without one (see ``_launch_allgather``); all other
  gathers are copy-engine transfers, one per shard. Backward: a hook on the
  unit's outputs gathers it again before its backward runs.
* Overlap (fused comm): reduce-scatters run on a communication stream as
  soon as a unit's gradients are complete, and while a unit's backward runs
  the next unit's parameters are gathered by the copy engines on a prefetch
  stream; the compute stream waits for the prefetch only when it needs the
  unit, and for the reduce-scatters only at the end of backward.
* Gradients: bf16 gradients are folded into a per-unit fp32 accumulator
  (exact across micro-steps); when a unit's gradients are complete on a
  syncing micro-step they are cast to bf16 into peer-mapped memory and
  reduce-scattered by ``nfb_rs_push`` (one kernel: bf16 cast of the fp32
  accumulator pushed to each slice's owner over NVLink, reduction in fp32,
  1/world scale, fp32 shard output), in a fixed unit order on every rank. With clipping off
  (``max_grad_norm`` <= 0) and ``final_backward`` set by the caller (the last
  backward before the optimizer step), ``nfb_rs_adamw`` instead applies AdamW
  to the shard inside the reduce-scatter (fp32 master, moments and the bf16
  shard the next all-gather reads), and the optimizer step has nothing left
  to do.
* The gradient norm for clipping is global: shard norms^2 are summed over ranks
  on the device (``nfb_allreduce_scalar``) before the update.

``comm="nccl"`` runs the same schedule on NCCL all_gather_into_tensor /
reduce_scatter_tensor (the baseline); ``comm="gloo"`` is the CPU test path.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch import nn

from .. import _native as nat
from ..profiling import trace
from .symm import SLOT_AG, SLOT_RS, SLOT_SCALAR, SymmetricWorkspace, symmetric_memory_available


def _round(n: int, a: int) -> int:
    return (n + a - 1) // a * a


@dataclass
class _Seg:
    name: str
    param: nn.Parameter
    start: int
    numel: int
    shape: torch.Size


@dataclass
class _Unit:
    index: int
    name: str
    module: nn.Module | None
    segs: list = field(default_factory=list)
    numel: int = 0
    shard: int = 0
    shard_start: int = 0       # offset of this unit's shard in the flat shard space
    full: torch.Tensor | None = None
    gathered: bool = False
    grad_off: int = -1         # peer-mapped bf16 full-gradient region (fused comm)
    acc32: torch.Tensor | None = None
    acc_fresh: bool = True
    pending: int = 0
    seen: set = field(default_factory=set)   # parameters whose gradient of this backward arrived
    ready: bool = False
    launched: bool = False
    bwd_gathered: bool = False
    prefix: int = 0            # elements of the leading 1-D parameters (copied ahead of a fused gather)
    ag_ok: bool = False        # the unit's first parameter consumer is a linear layer (fused gather allowed)
    ag_pending: bool = False   # storage allocated, prefix copied, the rest awaits the fused GEMM
    ready_event: object = None # prefetch all-gather in flight on the prefetch stream
    first_w: tuple | None = None   # (byte offset, bytes) of the weight the first linear consumes
    rest_event: object = None  # copy-engine gather of the unit minus first_w, in flight


class FullyShardedDataParallel(nn.Module):
    def __init__(self, module: nn.Module, param_dtype: torch.dtype | None = None, comm: str = "auto",
                 unit_types: tuple | None = None, reshard_after_forward: bool = True, ctas: int = 32,
                 process_group: dist.ProcessGroup | None = None, fuse_ag_gemm: bool | None = None,
                 fuse_rs_adamw: bool = True):
        super().__init__()
        self.module = module
        dev = next(module.parameters()).device
        self.device = dev
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.param_dtype = param_dtype or (torch.bfloat16 if dev.type == "cuda" else torch.float32)
        if comm == "auto":
            if dev.type != "cuda":
                comm = "gloo" if self.world > 1 else "none"
            else:
                comm = "fused" if (self.world > 1 and symmetric_memory_available()) else ("nccl" if self.world > 1
                                                                                          else "none")
        if comm == "fused" and self.param_dtype != torch.bfloat16:
            comm = "nccl"
        self.comm = comm
        self.reshard_after_forward = reshard_after_forward
        self.ctas = ctas
        if unit_types is None:
            from ..models.dit import DiTBlock
            from ..models.layers import TransformerBlock
            unit_types = (TransformerBlock, DiTBlock)
        self.units = self._build_units(unit_types)
        self.root = self.units[-1]
        from ..models.dit import DiTBlock
        from ..models.layers import TransformerBlock
        if fuse_ag_gemm is None:   # default on; NFB_FSDP_FUSE_AG=0 keeps the separate all-gather kernel
            import os
            fuse_ag_gemm = os.environ.get("NFB_FSDP_FUSE_AG", "1") != "0"
        self.fuse_ag_gemm = bool(fuse_ag_gemm and comm == "fused")
        for u in self.units[:-1]:
            # blocks whose first parameter use is a linear layer (after 1-D norm weights / biases)
            u.ag_ok = self.fuse_ag_gemm and isinstance(u.module, (TransformerBlock, DiTBlock))
        self._ag_unit: _Unit | None = None
        self.comm_stream = self.ag_stream = None
        if comm == "fused":
            self.comm_stream = torch.cuda.Stream(device=dev)
            self.ag_stream = torch.cuda.Stream(device=dev)
        self._ag_ready = torch.zeros(1024, dtype=torch.int32, device=dev) if self.fuse_ag_gemm else None
        self.ag_fused_launches = 0
        # Measured on B200: with one peer the in-kernel gather of the whole unit is as fast as
        # anything else; with more, every rank reads the consumed weight from the same one or two
        # owners, so the kernel gathers only that weight and the copy engines the rest.
        import os
        env = os.environ.get("NFB_FSDP_AG_HYBRID")
        self.ag_hybrid = (env == "1") if env is not None else self.world > 2
        self.fuse_rs_adamw = bool(fuse_rs_adamw and comm in ("fused", "gloo"))
        self._opt = None
        self._fused_updates = 0
        # clip phase 1 inside the reduce-scatters: per-CTA partials and the last-CTA ticket
        self._norm_units = 0
        self.norm_fused_steps = 0      # optimizer steps whose norm^2 came out of the reduce-scatters
        self.fuse_rs_norm = os.environ.get("NFB_FSDP_RS_NORM", "1") != "0"
        self._ss_partials = self._ss_ticket = None
        if comm == "fused":
            self._ss_partials = torch.zeros(256, dtype=torch.float32, device=dev)
            self._ss_ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        # Set by the caller (the Trainer does) when the coming backward is the last one before the
        # optimizer step: only then may AdamW run inside the reduce-scatter (with gradient
        # accumulation over several syncing backwards it would update on a partial gradient).
        self.final_backward = False
        self.fused_steps = 0           # optimizer steps applied inside the reduce-scatters
        self.shard_numel = sum(u.shard for u in self.units)
        self.master = torch.zeros(self.shard_numel, dtype=torch.float32, device=dev)
        self.grads = torch.zeros(self.shard_numel, dtype=torch.float32, device=dev)
        self.ws = None
        self.param_shards = None
        if comm == "fused":
            grad_bytes = sum(_round(u.numel * 2, 256) for u in self.units)
            self.ws = SymmetricWorkspace(_round(self.shard_numel * 2, 256) + grad_bytes + 4096, group=process_group,
                                         device=dev)
            self.param_off = self.ws.alloc(self.shard_numel * 2)
            for u in self.units:
                u.grad_off = self.ws.alloc(u.numel * 2)
        else:
            self.param_shards = torch.zeros(self.shard_numel, dtype=self.param_dtype, device=dev)
        self.params = self.param_shards
        self._init_shards()
        self._order: list[_Unit] = []       # reverse-backward (= forward) order of the current iteration
        self._rs_order: list[_Unit] = []
        self._next_rs = 0
        self.require_sync = True
        self._shard_fresh = True
        self._callback_queued = False
        self.comm_timer = None
        self._seg_of: dict[int, _Seg] = {}
        for u in self.units:
            for s in u.segs:
                s.param.register_post_accumulate_grad_hook(self._grad_hook)
                self._unit_of[id(s.param)] = u
                self._seg_of[id(s.param)] = s
                if s.param.dim() == 2:
                    # the native linear backward writes this weight's fp32 gradient straight into the
                    # unit's accumulator (grad_target / grad_done); autograd then receives none
                    s.param._nfb_grad_owner = self
        for u in self.units[:-1]:
            self._wrap_unit(u)
        self.module.register_forward_pre_hook(self._root_pre_forward)

    # ------------------------------------------------------------------ setup
    def _build_units(self, unit_types) -> list[_Unit]:
        self._unit_of: dict[int, _Unit] = {}
        units: list[_Unit] = []
        claimed: set[int] = set()

        def visit(mod: nn.Module, prefix: str):
            for name, child in mod.named_children():
                full = f"{prefix}{name}"
                if isinstance(child, unit_types):
                    units.append(self._make_unit(len(units), full, child, f"{full}."))
                    for p in child.parameters():
                        claimed.add(id(p))
                else:
                    visit(child, f"{full}.")

        visit(self.module, "")
        root = _Unit(len(units), "<root>", None)
        named = [(n, p) for n, p in self.module.named_parameters() if p.requires_grad and id(p) not in claimed]
        self._fill_unit(root, named)
        units.append(root)
        off = 0
        for u in units:
            u.shard_start = off
            off += u.shard
        return units

    def _make_unit(self, idx, name, module, prefix) -> _Unit:
        u = _Unit(idx, name, module)
        self._fill_unit(u, [(prefix + n, p) for n, p in module.named_parameters() if p.requires_grad])
        return u

    def _fill_unit(self, u: _Unit, named) -> None:
        # 1-D parameters first: they form the prefix a fused gather copies ahead
        named = [(n, p) for n, p in named if p.dim() <= 1] + [(n, p) for n, p in named if p.dim() > 1]
        off = 0
        for n, p in named:
            u.segs.append(_Seg(n, p, off, p.numel(), p.shape))
            off += _round(p.numel(), 8)
            if p.dim() <= 1:
                u.prefix = off
        u.numel = _round(max(off, 8), 8 * self.world)
        u.shard = u.numel // self.world
        u.pending = len(u.segs)

    def _init_shards(self) -> None:
        """Flatten each unit's initial fp32 parameters (rank 0's values), keep this rank's shard."""
        with torch.no_grad():
            for u in self.units:
                flat = torch.zeros(u.numel, dtype=torch.float32, device=self.device)
                for s in u.segs:
                    flat[s.start: s.start + s.numel].copy_(s.param.detach().reshape(-1).float())
                if self.world > 1:
                    dist.broadcast(flat, src=0, group=self.group)
                lo = self.rank * u.shard
                self.master[u.shard_start: u.shard_start + u.shard].copy_(flat[lo: lo + u.shard])
                u.full = torch.empty(u.numel, dtype=self.param_dtype, device=self.device)
                for s in u.segs:
                    s.param.data = u.full[s.start: s.start + s.numel].view(s.shape)
                u.full.untyped_storage().resize_(0)
            self._write_param_shards()

    def _write_param_shards(self) -> None:
        if self.comm == "fused":
            nat.call("nfb_cast", 0, 1, ctypes.c_void_p(self.ws.local_ptr(self.param_off)), nat.ptr(self.master),
                     self.shard_numel, 1.0, nat.stream(self.device))
            torch.cuda.synchronize(self.device)
        else:
            self.param_shards.copy_(self.master.to(self.param_dtype))

    # ------------------------------------------------------------ gather / reshard
    def _ensure_ready(self, u: _Unit) -> None:
        """Make the compute stream wait for a prefetch all-gather of ``u`` still in flight."""
        if u.ready_event is not None:
            main = torch.cuda.current_stream(self.device)
            if self.comm_timer is not None:   # time the compute stream stalls on the prefetch
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(main)
                main.wait_event(u.ready_event)
                e1.record(main)
                self.comm_timer.bracket(e0, e1)
            else:
                main.wait_event(u.ready_event)
            u.ready_event = None

    def _prefetch(self, u: _Unit) -> None:
        """Gather ``u`` on the prefetch stream (fused comm only)."""
        if u.gathered or self.comm != "fused" or u is self.root:
            return
        st = u.full.untyped_storage()
        nbytes = u.numel * u.full.element_size()
        if st.nbytes() != nbytes:
            st.resize_(nbytes)
        # the new storage may reuse memory the compute stream used until now
        self.ag_stream.wait_stream(torch.cuda.current_stream(self.device))
        self._launch_allgather(u, stream=self.ag_stream, barrier=False)
        ev = torch.cuda.Event()
        ev.record(self.ag_stream)
        u.ready_event = ev
        u.gathered = True

    def _gather(self, u: _Unit, lazy: bool = False) -> None:
        if u.gathered:
            self._ensure_ready(u)
            return
        with trace(f"fsdp.gather[{u.name}]"):
            self._gather_impl(u, lazy)

    def _gather_impl(self, u: _Unit, lazy: bool) -> None:
        if u.gathered:
            self._ensure_ready(u)
            return
        st = u.full.untyped_storage()
        nbytes = u.numel * u.full.element_size()
        if st.nbytes() != nbytes:
            st.resize_(nbytes)
        if lazy and u.ag_ok:
            self._copy_prefix(u)
            if u.first_w is not None and self.ag_hybrid:
                self._copy_rest(u)
            u.ag_pending = True
            u.gathered = True
            self._ag_unit = u
            from ..models import layers
            layers.set_pending_consumer(self._consume_linear)
            return
        # the root unit's gather opens each step's forward and carries the rank barrier
        self._launch_allgather(u, barrier=u is self.root)
        u.gathered = True

    def _launch_allgather(self, u: _Unit, stream: torch.cuda.Stream | None = None, slot: int = SLOT_AG,
                          barrier: bool = True) -> None:
        """Gather ``u`` into ``u.full``.

        Fused comm: with ``barrier`` the ``nfb_allgather`` kernel (rank barriers before and after the
        copy). Without it, one copy-engine transfer per shard and no SM use: valid for every gather
        after the first one of an optimizer step (the root unit's, which has the barrier), because
        a rank changes its shards only in its optimizer step or, with AdamW fused into the
        reduce-scatter, in the unit's reduce-scatter, whose own barrier every peer reaches only
        after its last gather of that unit.
        """
        if self.comm == "fused" and not barrier:
            sh = ctypes.c_void_p(stream.cuda_stream) if stream is not None else nat.stream(self.device)
            S = u.shard * 2
            src = self.param_off + u.shard_start * 2
            for i in range(self.world):
                q = (self.rank + i) % self.world
                nat.call("nfb_copy_async", ctypes.c_void_p(u.full.data_ptr() + q * S),
                         ctypes.c_void_p(self.ws.bases[q] + src), S, sh)
            return
        if self.comm == "fused":
            ws = self.ws
            sh = ctypes.c_void_p(stream.cuda_stream) if stream is not None else nat.stream(self.device)
            nat.call("nfb_allgather", ws.bases_ptr(), ws.rank, ws.world, u.shard,
                     self.param_off + u.shard_start * 2, nat.ptr(u.full), ws.flag_off, slot,
                     ws.next_epoch(slot), ws.timeout_ns, nat.ptr(ws.status), self.ctas, sh)
        elif self.comm == "nccl":
            dist.all_gather_into_tensor(u.full, self.param_shards[u.shard_start: u.shard_start + u.shard],
                                        group=self.group)
        elif self.comm == "gloo":
            parts = [torch.empty(u.shard, dtype=u.full.dtype, device=u.full.device) for _ in range(self.world)]
            dist.all_gather(parts, self.param_shards[u.shard_start: u.shard_start + u.shard].contiguous(),
                            group=self.group)
            u.full.copy_(torch.cat(parts))
        else:  # single process
            u.full.copy_(self.param_shards[u.shard_start: u.shard_start + u.shard])

    # ------------------------------------------------ all-gather fused into the first GEMM
    def _copy_prefix(self, u: _Unit) -> None:
        """Copy the unit's leading 1-D parameters from their owners (copy engine, over NVLink)."""
        end = u.prefix * 2
        if end == 0:
            return
        S = u.shard * 2
        src0 = self.param_off + u.shard_start * 2
        stream = nat.stream(self.device)
        for q in range(self.world):
            f0, f1 = q * S, min((q + 1) * S, end)
            if f1 <= f0:
                break
            nat.call("nfb_copy_async", ctypes.c_void_p(u.full.data_ptr() + f0),
                     ctypes.c_void_p(self.ws.bases[q] + src0), f1 - f0, stream)

    def _copy_rest(self, u: _Unit) -> None:
        """Copy-engine gather (prefetch stream) of the unit except its prefix and its first weight.

        The fused GEMM then gathers only the weight it consumes, so its NVLink volume is that
        weight's, and the copy engines move the other parameters at the same time.
        """
        src0 = self.param_off + u.shard_start * 2
        cs = self.ag_stream
        cs.wait_stream(torch.cuda.current_stream(self.device))   # the storage may be reused memory
        h = ctypes.c_void_p(cs.cuda_stream)
        for q, f0, f1 in rest_copies(u.prefix * 2, u.first_w, u.numel * 2, u.shard * 2, self.world, self.rank):
            nat.call("nfb_copy_async", ctypes.c_void_p(u.full.data_ptr() + f0),
                     ctypes.c_void_p(self.ws.bases[q] + src0 + (f0 - q * u.shard * 2)), f1 - f0, h)
        ev = torch.cuda.Event()
        ev.record(cs)
        u.rest_event = ev

    def _consume_linear(self, x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None):
        """The pending unit's first linear layer: run it as the all-gather-fused GEMM."""
        u = self._ag_unit
        if u is None or not u.ag_pending:
            return None
        full = u.full
        if w.untyped_storage().data_ptr() != full.untyped_storage().data_ptr():
            return None
        from ..models import layers
        u.ag_pending = False
        self._ag_unit = None
        layers.set_pending_consumer(None)
        K = x.shape[-1]
        off = w.data_ptr() - full.data_ptr()
        fits = (x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.dim() == 2 and w.is_contiguous()
                and K % 8 == 0 and x.numel() > 0 and off % 16 == 0
                and (w.shape[0] + 255) // 256 <= self._ag_ready.numel())
        if not fits:
            if u.rest_event is not None:
                torch.cuda.current_stream(self.device).wait_event(u.rest_event)
                u.rest_event = None
            self._launch_allgather(u, barrier=False)
            return None
        if u.first_w is None:
            u.first_w = (off, w.numel() * 2)   # later forwards gather the rest by copy engine
        y = _AgLinear.apply(x, w, self, u)
        if u.rest_event is not None:
            # every later use of the unit sees the copy-engine part too
            torch.cuda.current_stream(self.device).wait_event(u.rest_event)
            u.rest_event = None
        return y if b is None else y + b

    def _launch_ag_gemm(self, u: _Unit, x2: torch.Tensor, w: torch.Tensor, y: torch.Tensor) -> None:
        ws = self.ws
        M, K = x2.shape
        N = w.shape[0]
        off = w.data_ptr() - u.full.data_ptr()
        # with the rest of the unit in flight on the copy engines, gather only this weight (if this is
        # the weight those copies left out; otherwise the whole unit again, which rewrites equal bytes)
        only_w = u.rest_event is not None and u.first_w == (off, N * K * 2)
        lo, hi = (off, off + N * K * 2) if only_w else (u.prefix * 2, u.numel * 2)
        nat.call("nfb_ag_gemm", ws.bases_ptr(), ws.rank, ws.world, self.param_off + u.shard_start * 2, u.shard * 2,
                 nat.ptr(u.full), lo, hi, off, N, K, nat.ptr(x2),
                 x2.stride(0), M, nat.ptr(y), y.stride(0), nat.ptr(self._ag_ready), nat.ptr(ws.status),
                 nat.stream(self.device))
        self.ag_fused_launches += 1

    def _reshard(self, u: _Unit) -> None:
        if not u.gathered or u is self.root:
            return
        self._ensure_ready(u)   # no prefetch may still be writing the storage being released
        if u.rest_event is not None:
            torch.cuda.current_stream(self.device).wait_event(u.rest_event)
            u.rest_event = None
        u.full.untyped_storage().resize_(0)
        u.gathered = False

    # ------------------------------------------------------------------ hooks
    def _root_pre_forward(self, module, args):
        self._order = []
        self._gather(self.root)
        return None

    def _wrap_unit(self, u: _Unit) -> None:
        mod = u.module
        for meth in ("forward", "forward_chain"):
            fn = getattr(mod, meth, None)
            if fn is None:
                continue

            def wrapped(*a, _fn=fn, _u=u, **kw):
                self._pre_forward(_u)
                out = _fn(*a, **kw)
                self._post_forward(_u, out)
                return out

            setattr(mod, meth, wrapped)

    def _pre_forward(self, u: _Unit) -> None:
        # A unit recomputed in backward (activation checkpointing) is gathered in full: the
        # recompute has to replay the forward's ops, and the GEMM-fused gather exists only in the
        # forward (in backward the unit is gathered before its recompute).
        self._gather(u, lazy=self.fuse_ag_gemm and not getattr(u.module, "grad_checkpoint", False))
        if u not in self._order:
            self._order.append(u)
        u.bwd_gathered = False

    def _post_forward(self, u: _Unit, out) -> None:
        if u.ag_pending:
            raise RuntimeError(f"FSDP unit {u.name}: its deferred all-gather was never consumed by a linear layer")
        if torch.is_grad_enabled():
            for t in _tensors(out):
                if t.requires_grad:
                    t.register_hook(lambda g, _u=u: self._pre_backward(_u))
        if self.reshard_after_forward:
            self._reshard(u)

    def _pre_backward(self, u: _Unit) -> None:
        if not u.bwd_gathered:
            u.bwd_gathered = True
            self._gather(u)
            # the unit whose backward runs next (the previous one in forward order)
            i = self._order.index(u) if u in self._order else -1
            if i > 0 and not self._order[i - 1].bwd_gathered:
                self._prefetch(self._order[i - 1])

    def _grad_hook(self, p: nn.Parameter) -> None:
        if p.grad is None:
            return                 # its gradient went to grad_target, or it received none
        acc = self.grad_target(p)[0]
        acc.add_(p.grad.reshape(-1))
        p.grad = None
        self.grad_done(p)

    # gradient owner protocol (ops/linear.py:weight_grad): fp32 buffer + overwrite flag, then done
    def grad_target(self, p: nn.Parameter):
        """(``p``'s segment of its unit's fp32 gradient accumulator, overwrite?) for this backward."""
        if not self._callback_queued:
            self._callback_queued = True
            self._rs_order = list(reversed(self._order)) + [self.root]
            self._next_rs = 0
            torch.autograd.Variable._execution_engine.queue_callback(self._finalize_backward)
        u = self._unit_of[id(p)]
        if u.acc32 is None:
            u.acc32 = torch.zeros(u.numel, dtype=torch.float32, device=self.device)
        elif u.acc_fresh:
            u.acc32.zero_()      # new window: parameters without a gradient contribute zeros
        u.acc_fresh = False
        seg = self._seg_of[id(p)]
        return u.acc32[seg.start: seg.start + seg.numel], False

    def grad_done(self, p: nn.Parameter) -> None:
        """``p``'s gradient of this backward is in its unit's accumulator."""
        u = self._unit_of[id(p)]
        if id(p) in u.seen:
            raise RuntimeError(f"parameter {self._seg_of[id(p)].name} received a second gradient in one backward; "
                               "its unit may already be reduce-scattered")
        u.seen.add(id(p))
        u.pending -= 1
        if u.pending == 0:
            u.ready = True
            if self.require_sync:
                self._launch_ready()

    def _launch_ready(self) -> None:
        while self._next_rs < len(self._rs_order) and self._rs_order[self._next_rs].ready:
            u = self._rs_order[self._next_rs]
            self._reduce_scatter(u)
            self._next_rs += 1

    def _reduce_scatter(self, u: _Unit) -> None:
        with trace(f"fsdp.reduce_scatter[{u.name}]"):
            self._reduce_scatter_impl(u)

    def _reduce_scatter_impl(self, u: _Unit) -> None:
        u.launched = True
        if u.acc32 is None:
            u.acc32 = torch.zeros(u.numel, dtype=torch.float32, device=self.device)
        elif u.acc_fresh:
            u.acc32.zero_()      # no gradient reached this unit in the window
        out = self.grads[u.shard_start: u.shard_start + u.shard]
        scale = 1.0 / self.world
        if self.comm == "fused" and self._rs_adamw_active():
            ws, opt = self.ws, self._opt
            cs = self.comm_stream
            cs.wait_stream(torch.cuda.current_stream(self.device))
            hs = ctypes.c_void_p(cs.cuda_stream)
            # bf16 gradient into this rank's send region, then one kernel per unit: every rank pulls its slice
            # from all peers, reduces, scales and applies AdamW to its fp32 master / moments / bf16 shard
            nat.call("nfb_cast", 0, 1, ctypes.c_void_p(ws.local_ptr(u.grad_off)), nat.ptr(u.acc32), u.numel, 1.0, hs)
            lo, hi = u.shard_start, u.shard_start + u.shard
            b1, b2 = opt.betas
            nat.call("nfb_rs_adamw", ws.bases_ptr(), ws.rank, ws.world, u.shard, u.grad_off, ws.flag_off, SLOT_RS,
                     scale, ws.next_epoch(SLOT_RS), ws.timeout_ns, nat.ptr(ws.status), nat.ptr(self.master[lo:hi]),
                     nat.ptr(opt.m[lo:hi]), nat.ptr(opt.v[lo:hi]), self.param_off + u.shard_start * 2, opt.lr, b1, b2,
                     opt.eps, opt.weight_decay, opt.step_count + 1, 1.0, 1, self.ctas, hs)
            self._fused_updates += 1
        elif self.comm == "fused":
            ws = self.ws
            # on the communication stream, after the unit's gradients are complete on the compute stream
            cs = self.comm_stream
            cs.wait_stream(torch.cuda.current_stream(self.device))
            hs = ctypes.c_void_p(cs.cuda_stream)
            if self._rs_norm_active():
                # clip phase 1 fused into the reduce-scatter: each unit's kernel adds its shard's sum of
                # squares into the optimizer's norm^2 (zeroed on this stream before the first unit)
                opt = self._opt
                if self._norm_units == 0:
                    with torch.cuda.stream(cs):
                        opt.norm2.zero_()
                nat.call("nfb_rs_push_sumsq", ws.bases_ptr(), ws.rank, ws.world, nat.ptr(u.acc32), u.numel,
                         u.grad_off, ws.flag_off, SLOT_RS, scale, ws.next_epoch(SLOT_RS), ws.timeout_ns,
                         nat.ptr(ws.status), nat.ptr(out), 0, nat.ptr(self._ss_partials), nat.ptr(self._ss_ticket),
                         nat.ptr(opt.norm2), self.ctas, hs)
                self._norm_units += 1
            else:
                # one kernel: bf16 cast of the fp32 accumulator, pushed to the slice owners, reduced into the shard
                nat.call("nfb_rs_push", ws.bases_ptr(), ws.rank, ws.world, nat.ptr(u.acc32), u.numel, u.grad_off,
                         ws.flag_off, SLOT_RS, scale, ws.next_epoch(SLOT_RS), ws.timeout_ns, nat.ptr(ws.status),
                         nat.ptr(out), int(not self._shard_fresh), self.ctas, hs)
        elif self.comm == "nccl":
            red = torch.empty(u.shard, dtype=torch.bfloat16, device=self.device)
            dist.reduce_scatter_tensor(red, u.acc32.to(torch.bfloat16), group=self.group)
            if self._shard_fresh:
                out.copy_(red.float().mul_(scale))
            else:
                out.add_(red.float().mul_(scale))
        elif self.comm == "gloo":
            full = u.acc32.clone()
            dist.all_reduce(full, group=self.group)
            lo = self.rank * u.shard
            red = full[lo: lo + u.shard] * scale
            if self._rs_adamw_active():
                # same schedule as the fused device path: the shard's AdamW runs with its reduce-scatter
                self._adamw_shard(u.shard_start, u.shard_start + u.shard, red)
                self._fused_updates += 1
            elif self._shard_fresh:
                out.copy_(red)
            else:
                out.add_(red)
        else:
            if self._shard_fresh:
                out.copy_(u.acc32)
            else:
                out.add_(u.acc32)
        u.acc_fresh = True
        self._reshard(u)

    def _finalize_backward(self) -> None:
        self._callback_queued = False
        if self.require_sync:
            for u in self._rs_order:
                u.ready = True
            self._launch_ready()
            self._shard_fresh = False
        if self.comm_stream is not None:
            # the optimizer and the next window's accumulation wait for every reduce-scatter
            main = torch.cuda.current_stream(self.device)
            if self.comm_timer is not None and self.require_sync:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(main)
                main.wait_stream(self.comm_stream)
                e1.record(main)
                self.comm_timer.bracket(e0, e1)
            else:
                main.wait_stream(self.comm_stream)
        for u in self.units:
            u.pending = len(u.segs)
            u.seen = set()
            u.ready = False
            u.launched = False
            self._reshard(u)

    # ------------------------------------------------------------------ API
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

    def zero_grad(self) -> None:
        self._shard_fresh = True
        for u in self.units:
            u.acc_fresh = True

    def _norm_allreduce(self, norm2: torch.Tensor) -> None:
        if self.world == 1:
            return
        if self.comm == "fused":
            ws = self.ws
            nat.call("nfb_allreduce_scalar", ws.bases_ptr(), ws.rank, ws.world, ws.scalar_off, nat.ptr(norm2),
                     ws.flag_off, SLOT_SCALAR, ws.next_epoch(SLOT_SCALAR), ws.timeout_ns, nat.ptr(ws.status),
                     nat.stream(self.device))
        else:
            dist.all_reduce(norm2, group=self.group)

    def _after_step(self) -> None:
        if self.comm != "fused":
            self.param_shards.copy_(self.master.to(self.param_dtype))
        self.root.gathered = False   # the root unit is re-gathered by the next forward

    def make_optimizer(self, lr: float = 3e-4, weight_decay: float = 0.01, max_grad_norm: float = 1.0,
                       betas=(0.9, 0.999), eps: float = 1e-8):
        from ..optim.adamw import FlatAdamW

        ptr = self.ws.local_ptr(self.param_off) if self.comm == "fused" else None
        opt = FlatAdamW(self, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                        ddp=self, grads=self.grads, master=self.master,
                        params=None if ptr is not None else self.param_shards, params_ptr=ptr,
                        norm_allreduce=self._norm_allreduce, after_step=self._after_step)
        self._opt = opt
        opt.fused_owner = self
        return opt

    def _rs_norm_active(self) -> bool:
        """The reduce-scatters of this backward produce each shard's final gradient exactly once, with
        clipping on: their kernels can accumulate the global norm's sum of squares."""
        opt = self._opt
        return (opt is not None and self.require_sync and self.final_backward and self._shard_fresh
                and opt.max_grad_norm is not None and opt.max_grad_norm > 0 and self._ss_partials is not None
                and self.fuse_rs_norm)

    def take_norm2(self) -> bool:
        """True when every unit's reduce-scatter added its shard's sum of squares to the optimizer's norm^2
        this window (the optimizer then only sums it over ranks)."""
        n, self._norm_units = self._norm_units, 0
        if n == len(self.units):
            self.norm_fused_steps += 1
            return True
        return False

    def _rs_adamw_active(self) -> bool:
        opt = self._opt
        return (self.fuse_rs_adamw and opt is not None and self.require_sync and self.final_backward
                and self._shard_fresh and not (opt.max_grad_norm is not None and opt.max_grad_norm > 0))

    def _adamw_shard(self, lo: int, hi: int, g: torch.Tensor) -> None:
        """AdamW on shard elements [lo, hi) with gradient g (host path of the fused RS + AdamW)."""
        import math

        opt = self._opt
        b1, b2 = opt.betas
        step = opt.step_count + 1
        p, m, v = self.master[lo:hi], opt.m[lo:hi], opt.v[lo:hi]
        p.mul_(1 - opt.lr * opt.weight_decay)
        m.mul_(b1).add_(g, alpha=1 - b1)
        v.mul_(b2).addcmul_(g, g, value=1 - b2)
        denom = (v.sqrt() / math.sqrt(1 - b2 ** step)).add_(opt.eps)
        p.addcdiv_(m, denom, value=-opt.lr / (1 - b1 ** step))

    def take_fused_step(self) -> bool:
        """True when every unit's AdamW update already ran inside its reduce-scatter this window."""
        n, self._fused_updates = self._fused_updates, 0
        if n == 0:
            return False
        if n != len(self.units):
            raise RuntimeError(f"fused reduce-scatter + AdamW updated {n} of {len(self.units)} units")
        self.fused_steps += 1
        return True

    def check_health(self) -> None:
        if self.ws is not None:
            self.ws.check()

    # ------------------------------------------------------------- checkpoints
    def _full_flat_master(self, u: _Unit) -> torch.Tensor:
        shard = self.master[u.shard_start: u.shard_start + u.shard].contiguous()
        if self.world == 1:
            return shard.clone()
        if self.comm == "gloo":
            parts = [torch.empty_like(shard) for _ in range(self.world)]
            dist.all_gather(parts, shard, group=self.group)
            return torch.cat(parts)
        full = torch.empty(u.numel, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(full, shard, group=self.group)
        return full

    def full_master_views(self):
        """{id(param): full fp32 tensor} on rank 0 (collective; other ranks get None)."""
        views = {}
        for u in self.units:
            full = self._full_flat_master(u)
            if self.rank == 0:
                for s in u.segs:
                    views[id(s.param)] = full[s.start: s.start + s.numel].view(s.shape)
        return views if self.rank == 0 else None

    def load_full_state_dict(self, sd: dict) -> None:
        """Load a full reference-format state dict (every rank reads the same file)."""
        tmp = {id(s.param): torch.zeros(s.shape, dtype=torch.float32, device=self.device)
               for u in self.units for s in u.segs}
        saved = {}
        for u in self.units:
            for s in u.segs:
                saved[id(s.param)] = s.param.data
                s.param.data = tmp[id(s.param)]
        try:
            self.module.load_state_dict(sd, strict=True)
        finally:
            for u in self.units:
                for s in u.segs:
                    s.param.data = saved[id(s.param)]
        with torch.no_grad():
            for u in self.units:
                flat = torch.zeros(u.numel, dtype=torch.float32, device=self.device)
                for s in u.segs:
                    flat[s.start: s.start + s.numel].copy_(tmp[id(s.param)].reshape(-1))
                lo = self.rank * u.shard
                self.master[u.shard_start: u.shard_start + u.shard].copy_(flat[lo: lo + u.shard])
        self._write_param_shards()
        self.root.gathered = False

    def gather_optimizer_state(self, opt) -> dict:
        """Optimizer moments of every rank's shard, collected on rank 0 (same world size to resume)."""
        m, v = opt.m.contiguous(), opt.v.contiguous()
        if self.world > 1:
            ms = [torch.empty_like(m) for _ in range(self.world)]
            vs = [torch.empty_like(v) for _ in range(self.world)]
            dist.all_gather(ms, m, group=self.group)
            dist.all_gather(vs, v, group=self.group)
        else:
            ms, vs = [m], [v]
        return {"step": opt.step_count, "world": self.world, "exp_avg_shards": [t.cpu() for t in ms],
                "exp_avg_sq_shards": [t.cpu() for t in vs]}

    def load_optimizer_state(self, opt, sd: dict) -> None:
        if sd.get("world") != self.world:
            raise ValueError(f"optimizer state was saved with world={sd.get('world')}, running world={self.world}")
        opt.step_count = int(sd["step"])
        opt.m.copy_(sd["exp_avg_shards"][self.rank].to(opt.m.device))
        opt.v.copy_(sd["exp_avg_sq_shards"][self.rank].to(opt.v.device))


def rest_copies(prefix_bytes: int, first_w: tuple, total_bytes: int, shard_bytes: int, world: int, rank: int):
    """Copy-engine transfers (owner, flat byte start, end) for a unit minus its prefix and first weight.

    The flat range [prefix_bytes, total_bytes) without [w0, w0 + wbytes) is split at shard
    boundaries; owners are visited from rank+1 on, so ranks start on different peers.
    """
    w0, w1 = first_w[0], first_w[0] + first_w[1]
    out = []
    for i in range(world):
        q = (rank + 1 + i) % world
        for lo, hi in ((prefix_bytes, w0), (w1, total_bytes)):
            f0, f1 = max(lo, q * shard_bytes), min(hi, (q + 1) * shard_bytes)
            if f1 > f0:
                out.append((q, f0, f1))
    return out


class _AgLinear(torch.autograd.Function):
    """y = x @ w.T where the forward GEMM also gathers w's FSDP unit (``nfb_ag_gemm``).

    Backward runs after the unit was gathered again, with plain GEMMs.
    """

    @staticmethod
    def forward(ctx, x, w, fsdp, u):
        K = x.shape[-1]
        x2 = x.reshape(-1, K)
        if not x2.is_contiguous() or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        y = torch.empty((x2.shape[0], w.shape[0]), dtype=x.dtype, device=x.device)
        fsdp._launch_ag_gemm(u, x2, w, y)
        ctx.save_for_backward(x, w)
        ctx.w_ref = w          # the Parameter itself: its gradient owner is an attribute
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        from ..ops import linear as linear_op

        x, w = ctx.saved_tensors
        gy2 = gy.reshape(-1, gy.shape[-1])
        x2 = x.reshape(-1, x.shape[-1])
        native = linear_op.supported(x2, w)
        if native:
            gy2, x2 = linear_op._aligned_rows(gy2), linear_op._aligned_rows(x2)
        gx = gw = None
        if ctx.needs_input_grad[0]:
            gx = (linear_op.input_grad(gy2, w) if native else gy2 @ w).view(x.shape)
        if ctx.needs_input_grad[1]:
            gw = linear_op.weight_grad(gy2, x2, ctx.w_ref) if native else gy2.t() @ x2
        return gx, gw, None, None


def _tensors(obj):
    if isinstance(obj, torch.Tensor):
        yield obj
    elif isinstance(obj, (tuple, list)):
        for o in obj:
            yield from _tensors(o)
    elif isinstance(obj, dict):
        for o in obj.values():
            yield from _tensors(o)
