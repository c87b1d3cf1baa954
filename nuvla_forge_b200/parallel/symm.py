"""Symmetric device memory for the fused NVLink collectives.

One buffer of the same size on every rank, mapped into every peer's address
space by PyTorch's symmetric-memory rendezvous (CUDA VMM + IPC handles
exchanged through the process group's store). The native kernels (csrc/comm.cu)
receive every rank's base pointer and address peers with plain loads and
stores over NVLink.

Layout (byte offsets): [flags | scalar exchange | data ...]. ``alloc`` hands
out 256-byte-aligned regions of the data area at construction time (callers
reserve what they need up front; every rank must reserve the same sequence).

Each collective kind uses its own flag *slot*; every launch takes the next
epoch of its slot (a host counter that all ranks advance identically, because
all ranks launch the same collectives in the same order). Bounded waits in
the kernels report into ``status``; :meth:`check` raises ``CommTimeout``.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from .. import _native as nat

SLOT_DDP, SLOT_RS, SLOT_AG, SLOT_SCALAR, SLOT_TEST = 0, 1, 2, 3, 4


class CommTimeout(RuntimeError):
    """A fused collective gave up waiting for a peer (the peer died or stalled)."""


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


def decode_status(v: int) -> str:
    code, where = (v >> 24) & 0xFF, v & 0xFFFFFF
    kinds = {1: "barrier timeout", 2: "flag timeout", 3: "bad argument"}
    return f"{kinds.get(code, f'code {code}')} at site {where & 0xFFFF} (peer {where >> 16})"


class SymmetricWorkspace:
    def __init__(self, data_bytes: int, group: dist.ProcessGroup | None = None,
                 device: torch.device | None = None, timeout_s: float | None = None):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group or dist.group.WORLD
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.flag_off = 0
        self.scalar_off = _align(int(nat.lib().nfb_comm_flag_bytes()))
        self.data_off = self.scalar_off + 256
        self.total = self.data_off + _align(max(int(data_bytes), 256))
        self.buf = symm_mem.empty(self.total, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        torch.cuda.synchronize(self.device)
        try:
            self.handle = symm_mem.rendezvous(self.buf, self.group)
        except Exception:  # older API wants the group enabled first
            symm_mem.enable_symm_mem_for_group(self.group.group_name)
            self.handle = symm_mem.rendezvous(self.buf, self.group.group_name)
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.bases = (ctypes.c_uint64 * self.world)(*ptrs)
        self.multicast_ptr = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        self._cursor = self.data_off
        self.epochs = [0] * 8
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        t = timeout_s if timeout_s is not None else float(os.environ.get("NFB_COMM_TIMEOUT_S", "30"))
        self.timeout_ns = int(t * 1e9)
        dist.barrier(self.group)

    def alloc(self, nbytes: int) -> int:
        """Reserve ``nbytes`` of the data area; returns the region's byte offset."""
        off = self._cursor
        end = off + _align(nbytes)
        if end > self.total:
            raise MemoryError(f"symmetric workspace exhausted ({end} > {self.total} bytes)")
        self._cursor = end
        return off

    def local_view(self, off: int, numel: int, dtype: torch.dtype) -> torch.Tensor:
        es = torch.empty((), dtype=dtype).element_size()
        return self.buf[off: off + numel * es].view(dtype)

    def next_epoch(self, slot: int) -> int:
        self.epochs[slot] = (self.epochs[slot] + 1) & 0x7FFFFFFF
        return self.epochs[slot]

    def bases_ptr(self) -> ctypes.c_void_p:
        return ctypes.cast(self.bases, ctypes.c_void_p)

    def check(self) -> None:
        v = int(self.status.item())
        if v:
            raise CommTimeout(f"rank {self.rank}: fused collective failed: {decode_status(v)}")


def symmetric_memory_available() -> bool:
    if not (torch.cuda.is_available() and nat.HAS_NATIVE and dist.is_initialized()):
        return False
    try:
        import torch.distributed._symmetric_memory  # noqa: F401
    except Exception:  # noqa: BLE001
        return False
    return dist.get_world_size() <= 8
